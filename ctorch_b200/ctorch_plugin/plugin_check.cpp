// plugin_check.cpp — drives ctorch's public API on CUDA tensors with the B200 backend linked in
// (cuda_backend.cpp) and compares every result with ctorch's own CPU path on the same inputs.
//   plugin_check --registry   every CUDA dispatch slot is filled (needs no GPU)
//   plugin_check              the ops on cuda:0 vs CPU (bit-exact, float sums to 1e-5 relative)
//   plugin_check --bench      device time of the hot-path ops through ctorch's API on cuda:0,
//                             one JSON line per (op, path); see bench() below
#include "ctorch/dispatch.h"
#include "ctorch/errors.h"
#include "ctorch/ops/elementwise.h"
#include "ctorch/ops/indexing.h"
#include "ctorch/ops/op_keys.h"
#include "ctorch/ops/reduction.h"
#include "ctorch/tensor.h"

#include "b200_cast.h"
#include "ops/cast_cpu.h"
#include "ops/reduction.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <string>
#include <vector>

using namespace ctorch;

namespace {

int g_pass = 0, g_fail = 0;

void report(bool ok, const std::string& what) {
    if (ok) {
        ++g_pass;
    } else {
        ++g_fail;
        std::printf("FAIL %s\n", what.c_str());
    }
}

uint64_t g_state = 0x243F6A8885A308D3ULL;
uint64_t next_u64() {
    g_state += 0x9E3779B97F4A7C15ULL;
    uint64_t z = g_state;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

Tensor make(std::vector<int64_t> shape, dtype dt, bool small_ints = false) {
    Tensor t(shape, dt, Device::cpu());
    const int64_t n = t.numel();
    void* p = t.storage().data();
    for (int64_t i = 0; i < n; ++i) {
        const uint64_t h = next_u64();
        const double u = static_cast<double>(h >> 11) * 0x1.0p-53 * 2.0 - 1.0;
        switch (dt) {
        case dtype::float32: static_cast<float*>(p)[i] = static_cast<float>(u * 3); break;
        case dtype::float64: static_cast<double*>(p)[i] = u * 3; break;
        case dtype::int32: static_cast<int32_t*>(p)[i] = small_ints ? static_cast<int32_t>(h % 7) : static_cast<int32_t>(h % 2001) - 1000; break;
        case dtype::int64: static_cast<int64_t*>(p)[i] = small_ints ? static_cast<int64_t>(h % 7) : static_cast<int64_t>(h % 2001) - 1000; break;
        case dtype::bool_: static_cast<unsigned char*>(p)[i] = static_cast<unsigned char>(h & 1); break;
        default: break;
        }
    }
    return t;
}

std::vector<unsigned char> bytes_of(const Tensor& t) {
    Tensor c = t.device().is_cpu() ? t.contiguous() : t.to(Device::cpu()).contiguous();
    const std::size_t es = size_of(c.dtype());
    const std::size_t n = static_cast<std::size_t>(c.numel()) * es;
    std::vector<unsigned char> out(n);
    if (n) std::memcpy(out.data(), static_cast<const char*>(c.storage().data()) + c.offset() * es, n);
    return out;
}

bool same_bits(const Tensor& gpu, const Tensor& cpu) {
    return gpu.shape() == cpu.shape() && gpu.dtype() == cpu.dtype() && bytes_of(gpu) == bytes_of(cpu);
}

bool close(const Tensor& gpu, const Tensor& cpu, double tol) {
    if (gpu.shape() != cpu.shape() || gpu.dtype() != cpu.dtype()) return false;
    Tensor g = gpu.to(Device::cpu()).contiguous();
    Tensor c = cpu.contiguous();
    const int64_t n = c.numel();
    for (int64_t i = 0; i < n; ++i) {
        double gv, cv;
        if (c.dtype() == dtype::float32) {
            gv = static_cast<const float*>(g.storage().data())[i];
            cv = static_cast<const float*>(c.storage().data())[c.offset() + i];
        } else {
            gv = static_cast<const double*>(g.storage().data())[i];
            cv = static_cast<const double*>(c.storage().data())[c.offset() + i];
        }
        if (std::isnan(cv) != std::isnan(gv)) return false;
        if (!std::isnan(cv) && std::fabs(gv - cv) > tol * std::max(1.0, std::fabs(cv))) return false;
    }
    return true;
}

template <class E> bool throws(const std::function<void()>& f) {
    try {
        f();
    } catch (const E&) {
        return true;
    } catch (...) {
        return false;
    }
    return false;
}

int registry() {
    int missing = 0;
    auto need = [&](bool ok, const char* name) {
        if (!ok) {
            std::printf("missing CUDA slot %s\n", name);
            ++missing;
        }
    };
    const auto K = Device::Kind::CUDA;
    need(dispatch::has_op<op::AddOp>(K), "AddOp");
    need(dispatch::has_op<op::SubOp>(K), "SubOp");
    need(dispatch::has_op<op::MulOp>(K), "MulOp");
    need(dispatch::has_op<op::DivOp>(K), "DivOp");
    need(dispatch::has_op<op::AddInplaceOp>(K), "AddInplaceOp");
    need(dispatch::has_op<op::SubInplaceOp>(K), "SubInplaceOp");
    need(dispatch::has_op<op::MulInplaceOp>(K), "MulInplaceOp");
    need(dispatch::has_op<op::DivInplaceOp>(K), "DivInplaceOp");
    need(dispatch::has_op<op::NegOp>(K), "NegOp");
    need(dispatch::has_op<op::AbsOp>(K), "AbsOp");
    need(dispatch::has_op<op::ExpOp>(K), "ExpOp");
    need(dispatch::has_op<op::LogOp>(K), "LogOp");
    need(dispatch::has_op<op::SqrtOp>(K), "SqrtOp");
    need(dispatch::has_op<op::ReluOp>(K), "ReluOp");
    need(dispatch::has_op<op::SigmoidOp>(K), "SigmoidOp");
    need(dispatch::has_op<op::TanhOp>(K), "TanhOp");
    need(dispatch::has_op<op::SumOp>(K), "SumOp");
    need(dispatch::has_op<op::MeanOp>(K), "MeanOp");
    need(dispatch::has_op<op::ProdOp>(K), "ProdOp");
    need(dispatch::has_op<op::MaxValOp>(K), "MaxValOp");
    need(dispatch::has_op<op::MinValOp>(K), "MinValOp");
    need(dispatch::has_op<op::MaxValIdxOp>(K), "MaxValIdxOp");
    need(dispatch::has_op<op::MinValIdxOp>(K), "MinValIdxOp");
    need(dispatch::has_op<op::ArgmaxOp>(K), "ArgmaxOp");
    need(dispatch::has_op<op::ArgminOp>(K), "ArgminOp");
    need(dispatch::has_op<op::IndexSelectOp>(K), "IndexSelectOp");
    std::printf("registry: %d of 26 CUDA slots filled\n", 26 - missing);
    return missing ? 1 : 0;
}

// ---- --bench: the hot-path ops through ctorch's own API on cuda:0 ----
//
// Three paths per op:
//   dispatch    dispatch::call<Op>(Device::Kind::CUDA, ...) into preallocated outputs: ctorch's
//               dispatcher, this backend's C++ shim and its kernels, the pattern of ctorch's own
//               benchmark (tests/bench/add_bench.cpp:79-90);
//   front_door  the public function (ctorch::add, ctorch::sum, ...): the same plus the output's
//               allocation through ctorch's caching allocator and the zero-fill its Storage does
//               on construction (src/storage.cpp:33-56);
//   zero_fill   that zero-fill alone (cudaMemset of the output's bytes), i.e. what an opt-in
//               uninitialised Storage would take off the front door.
// `us` is the mean device time per call over `reps` calls back to back between CUDA events on the
// legacy stream (the stream the backend launches on); `host_us` is the host time per call of that
// loop (when it reaches `us`, the host, not the GPU, sets the pace); `us_sync` is ctorch's own
// measure, the median host time of one call between two cudaDeviceSynchronize (so it includes
// the launch latency). Configuration 1's inputs are used as 4 copies in turn (536 MB > the 126 MB L2); the
// others exceed L2 on their own.

double now_s() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

template <class F> void time_path(const char* cfg, const char* op, const char* path, double bytes, int reps, F&& f) {
    for (int i = 0; i < 3; ++i) f(i);
    cudaDeviceSynchronize();
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventRecord(e0, cudaStreamLegacy);
    const double h0 = now_s();
    for (int i = 0; i < reps; ++i) f(i);
    const double host_us = (now_s() - h0) * 1e6 / reps;
    cudaEventRecord(e1, cudaStreamLegacy);
    cudaEventSynchronize(e1);
    float ms = 0.f;
    cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    std::vector<double> ts;
    for (int i = 0; i < std::min(reps, 25); ++i) {
        cudaDeviceSynchronize();
        const double t0 = now_s();
        f(i);
        cudaDeviceSynchronize();
        ts.push_back(now_s() - t0);
    }
    std::sort(ts.begin(), ts.end());
    const double us = ms * 1e3 / reps;
    const cudaError_t err = cudaGetLastError();
    std::printf("{\"config\": \"%s\", \"op\": \"%s\", \"path\": \"%s\", \"us\": %.3f, \"us_sync\": %.3f, "
                "\"host_us\": %.3f, \"gbs\": %.1f, \"algorithmic_bytes\": %.0f, \"reps\": %d, \"cuda\": \"%s\"}\n",
                cfg, op, path, us, ts[ts.size() / 2] * 1e6, host_us, bytes / (us * 1e-6) / 1e9, bytes, reps,
                cudaGetErrorString(err));
    std::fflush(stdout);
}

int bench(int reps) {
    const Device gpu = Device::cuda(0);
    const auto K = Device::Kind::CUDA;
    {  // configuration 1: add [4096,4096] + [1,4096], relu
        const int64_t n = 4096;
        std::vector<Tensor> A, B, C, O;
        for (int c = 0; c < 4; ++c) {
            A.push_back(make({n, n}, dtype::float32).to(gpu));
            B.push_back(make({1, n}, dtype::float32).to(gpu));
            C.push_back(add(A.back(), B.back()));
            O.push_back(Tensor({n, n}, dtype::float32, gpu));
        }
        const double add_b = 2.0 * n * n * 4 + n * 4, relu_b = 2.0 * n * n * 4;
        time_path("1", "add", "dispatch", add_b, reps, [&](int i) { dispatch::call<op::AddOp>(K, A[i & 3], B[i & 3], O[i & 3]); });
        time_path("1", "add", "front_door", add_b, reps, [&](int i) { (void)add(A[i & 3], B[i & 3]); });
        time_path("1", "relu", "dispatch", relu_b, reps, [&](int i) { dispatch::call<op::ReluOp>(K, C[i & 3], O[i & 3]); });
        time_path("1", "relu", "front_door", relu_b, reps, [&](int i) { (void)relu(C[i & 3]); });
        time_path("1", "[4096,4096] float32 output", "zero_fill", n * n * 4.0, reps,
                  [&](int i) { cudaMemset(O[i & 3].storage().data(), 0, n * n * 4); });
    }
    {  // configuration 2: X [8192,8192]: sum/mean over dim 1 (keepdim), max/argmax over dim 0, prod dim 1
        const int64_t n = 8192;
        Tensor X = make({n, n}, dtype::float32).to(gpu);
        Tensor s1({n, 1}, dtype::float32, gpu), v0({n}, dtype::float32, gpu), i0({n}, dtype::int64, gpu);
        const ops::ReductionAxes ax1 = ops::canonicalise(X, {1});
        const std::vector<int64_t> d1{1};
        const double rd = double(n) * n * 4;
        time_path("2", "sum dim=1 keepdim", "dispatch", rd + n * 4, reps, [&](int) { dispatch::call<op::SumOp>(K, X, s1, ax1); });
        time_path("2", "sum dim=1 keepdim", "front_door", rd + n * 4, reps, [&](int) { (void)sum(X, d1, true); });
        time_path("2", "mean dim=1 keepdim", "dispatch", rd + n * 4, reps, [&](int) { dispatch::call<op::MeanOp>(K, X, s1, ax1); });
        time_path("2", "max dim=0 (values+indices)", "dispatch", rd + n * 12, reps,
                  [&](int) { dispatch::call<op::MaxValIdxOp>(K, X, v0, i0, 0); });
        time_path("2", "max dim=0 (values+indices)", "front_door", rd + n * 12, reps, [&](int) { (void)ctorch::max(X, int64_t{0}, false); });
        time_path("2", "argmax dim=0", "dispatch", rd + n * 8, reps, [&](int) { dispatch::call<op::ArgmaxOp>(K, X, i0, 0); });
        time_path("2", "argmax dim=0", "front_door", rd + n * 8, reps, [&](int) { (void)argmax(X, 0); });
    }
    {  // configuration 4: int32 [64,512,1024] * transpose(1,2) of float32 [64,1024,512]; / float64 [1,512,1]
        Tensor I = make({64, 512, 1024}, dtype::int32).to(gpu);
        Tensor F = make({64, 1024, 512}, dtype::float32).to(gpu);
        Tensor D = make({1, 512, 1}, dtype::float64).to(gpu);
        Tensor Ft = F.permute({0, 2, 1});
        Tensor P({64, 512, 1024}, dtype::float32, gpu), Q({64, 512, 1024}, dtype::float64, gpu);
        const double e = 64.0 * 512 * 1024;
        // mixed operand dtypes reach the backend only through dispatch::call: ctorch's front-door
        // casts first, on the host (src/ops/binary_ops_cpu.cpp:154-184)
        time_path("4", "mul int32 x float32^T -> float32", "dispatch", e * 12, reps,
                  [&](int) { dispatch::call<op::MulOp>(K, I, Ft, P); });
        time_path("4", "div float32 / float64[1,512,1] -> float64", "dispatch", e * 12 + 4096, reps,
                  [&](int) { dispatch::call<op::DivOp>(K, P, D, Q); });
    }
    {  // configuration 3: index_select of 4194304 rows from a float32 [1000000, 256] table
        Tensor T = make({1000000, 256}, dtype::float32).to(gpu);
        Tensor idx({4194304}, dtype::int64, Device::cpu());
        auto* ip = static_cast<int64_t*>(idx.storage().data());
        for (int64_t i = 0; i < 4194304; ++i) ip[i] = static_cast<int64_t>(next_u64() % 1000000);
        Tensor ig = idx.to(gpu), out({4194304, 256}, dtype::float32, gpu);
        const double b = 4194304.0 * 8 + 2.0 * 4194304 * 256 * 4;
        const int r3 = std::max(3, reps / 10);
        time_path("3", "index_select float32", "dispatch", b, r3, [&](int) { dispatch::call<op::IndexSelectOp>(K, T, 0, ig, out); });
        time_path("3", "index_select float32", "front_door", b, r3, [&](int) { (void)index_select(T, 0, ig); });
        time_path("3", "[4194304,256] float32 output", "zero_fill", 4194304.0 * 256 * 4, r3,
                  [&](int) { cudaMemset(out.storage().data(), 0, size_t(4194304) * 256 * 4); });
    }
    return cudaDeviceSynchronize() == cudaSuccess ? 0 : 1;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc > 1 && std::strcmp(argv[1], "--registry") == 0) return registry();
    if (argc > 1 && std::strcmp(argv[1], "--bench") == 0) return bench(argc > 2 ? std::atoi(argv[2]) : 50);
    const Device gpu = Device::cuda(0);

    // elementwise, broadcast and views
    Tensor A = make({64, 256}, dtype::float32), B = make({1, 256}, dtype::float32);
    report(same_bits(add(A.to(gpu), B.to(gpu)), add(A, B)), "add broadcast");
    report(same_bits(relu(add(A.to(gpu), B.to(gpu))), relu(add(A, B))), "relu(add)");
    Tensor P = make({256, 64}, dtype::float32);
    report(same_bits(mul(A.to(gpu), P.to(gpu).permute({1, 0})), mul(A, P.permute({1, 0}))), "mul permuted rhs");
    report(same_bits(sub(A.to(gpu).slice(1, 1, 256, 3), B.to(gpu).slice(1, 0, 255, 3)),
                     sub(A.slice(1, 1, 256, 3), B.slice(1, 0, 255, 3))), "sub strided slices");
    report(same_bits(div(A.to(gpu), B.to(gpu)), div(A, B)), "div");
    Tensor I = make({64, 256}, dtype::int32), D = make({1, 256}, dtype::float64);
    report(same_bits(mul(I.to(gpu), A.to(gpu)), mul(I, A)), "mul int32*float32 (promotion)");
    report(same_bits(div(A.to(gpu), D.to(gpu)), div(A, D)), "div float32/float64 (promotion)");
    report(same_bits(add(I.to(gpu), I.to(gpu)), add(I, I)), "add int32");
    report(throws<DTypeError>([&] { div(I.to(gpu), I.to(gpu)); }), "integer div throws DTypeError");
    Tensor Ag = A.to(gpu), Ac = A.contiguous();
    Tensor Acopy = A.to(Device::cpu());
    add_(Ag, B.to(gpu));
    Tensor Ac2 = make({64, 256}, dtype::float32);
    std::memcpy(Ac2.storage().data(), A.storage().data(), 64 * 256 * 4);
    add_(Ac2, B);
    report(same_bits(Ag, Ac2), "add_ in place");
    using UFn = Tensor (*)(const Tensor&);
    const struct {
        UFn f;
        bool exact;
        const char* name;
    } unary_ops[] = {{&ctorch::neg, true, "neg"},   {&ctorch::abs, true, "abs"},
                     {&ctorch::exp, false, "exp"},  {&ctorch::log, false, "log"},
                     {&ctorch::sqrt, true, "sqrt"}, {&ctorch::sigmoid, false, "sigmoid"},
                     {&ctorch::tanh, false, "tanh"}};
    const Tensor pos = ctorch::abs(A);
    for (const auto& u : unary_ops) {
        Tensor g = u.f(pos.to(gpu)), c = u.f(pos);
        report(u.exact ? same_bits(g, c) : close(g, c, 2e-6), u.name);
    }

    // reductions
    Tensor X = make({300, 1000}, dtype::float32);
    const std::vector<int64_t> d0{0}, d1{1}, d01{0, 1};
    report(close(sum(X.to(gpu), d1, true), sum(X, d1, true), 1e-5), "sum dim1 keepdim");
    report(close(mean(X.to(gpu), d1, true), mean(X, d1, true), 1e-5), "mean dim1 keepdim");
    report(close(sum(X.to(gpu)), sum(X), 1e-5), "sum whole");
    report(close(sum(X.to(gpu), d0), sum(X, d0), 1e-5), "sum dim0");
    Tensor Xp({300, 1000}, dtype::float32, Device::cpu());
    for (int64_t i = 0; i < Xp.numel(); ++i)
        static_cast<float*>(Xp.storage().data())[i] = 1.0f + 0.001f * static_cast<const float*>(X.storage().data())[i];
    report(close(prod(Xp.to(gpu), std::vector<int64_t>{1}), prod(Xp, std::vector<int64_t>{1}), 1e-5), "prod dim1");
    report(same_bits(ctorch::max(X.to(gpu)), ctorch::max(X)), "max whole");
    report(same_bits(ctorch::min(X.to(gpu), std::vector<int64_t>{0}, false),
                     ctorch::min(X, std::vector<int64_t>{0}, false)), "min dim0 values");
    {
        auto g = ctorch::max(X.to(gpu), int64_t{0}, false);
        auto c = ctorch::max(X, int64_t{0}, false);
        report(same_bits(g.values, c.values) && same_bits(g.indices, c.indices), "max dim0 with indices");
    }
    Tensor T = make({500, 400}, dtype::int32, true);  // many ties
    report(same_bits(argmax(T.to(gpu), 0), argmax(T, 0)), "argmax ties dim0");
    report(same_bits(argmin(T.to(gpu), 1, true), argmin(T, 1, true)), "argmin ties dim1");
    report(same_bits(sum(T.to(gpu), d01), sum(T, d01)), "sum int32 -> int64");
    report(throws<ShapeError>([&] { ctorch::max(make({3, 0}, dtype::float32).to(gpu), std::vector<int64_t>{1}); }),
           "max over empty slice throws");

    // index_select
    Tensor idx({5}, dtype::int64, Device::cpu());
    const int64_t iv[5] = {3, -1, 0, 299, 3};
    std::memcpy(idx.storage().data(), iv, sizeof(iv));
    report(same_bits(index_select(X.to(gpu), 0, idx.to(gpu)), index_select(X, 0, idx)), "index_select rows");
    report(same_bits(index_select(X.to(gpu), 1, idx.to(gpu)), index_select(X, 1, idx)), "index_select columns");
    Tensor bad({1}, dtype::int64, Device::cpu());
    const int64_t bv = 300;
    std::memcpy(bad.storage().data(), &bv, sizeof(bv));
    report(throws<ShapeError>([&] { index_select(X.to(gpu), 0, bad.to(gpu)); }), "index_select out of range throws");

    // device-side cast and contiguous (b200_cast.h) vs ctorch's CPU cast
    {
        const dtype dts[] = {dtype::float32, dtype::float64, dtype::int32, dtype::int64, dtype::bool_};
        for (dtype from : dts) {
            Tensor src = make({37, 53}, from);
            Tensor view_g = src.to(gpu).permute(std::vector<int64_t>{1, 0});
            Tensor view_c = src.permute(std::vector<int64_t>{1, 0});
            for (dtype to : dts) {
                Tensor g = b200::cast_cuda(view_g, to);
                report(g.is_contiguous() && same_bits(g, ops::cast_cpu(view_c.contiguous(), to)),
                       std::string("cast ") + std::to_string(static_cast<int>(from)) + "->" +
                           std::to_string(static_cast<int>(to)));
            }
            report(same_bits(b200::contiguous_cuda(view_g), view_c.contiguous()), "contiguous_cuda");
        }
        report(throws<DTypeError>([&] { b200::cast_cuda(X.to(gpu), dtype::bfloat16); }), "cast to bfloat16 throws");
    }

    std::printf("plugin_check: %d passed, %d failed\n", g_pass, g_fail);
    return g_fail ? 1 : 0;
}
