// cuda_backend.cpp — ctorch's CUDA backend, re-implemented on the B200 C ABI (include/ctb/ctb.h).
//
// ctorch's CPU registrars call four extern "C" hooks at static-init time to fill the CUDA slots
// of its dispatch table (src/ops/binary_ops_cpu.cpp:130,146, unary_ops_cpu.cpp:126,142,
// reduction_ops_cpu.cpp:371,388, indexing_cpu.cpp:144,153). This file defines those four hooks;
// linked into ctorch in place of src/ops/*_cuda.cu it makes every ctorch CUDA op run on the
// sm_100a kernels. Every backend function keeps the contract of the slot it fills
// (include/ctorch/ops/op_keys.h): outputs are preallocated by ctorch's front-door, inputs may be
// strided views with an element offset, work runs on the legacy default stream under a
// DeviceGuard for the output's device (as ctorch's own CUDA kernels do,
// src/ops/binary_ops_cuda.cu:88), scratch comes from ctorch's per-device caching allocator
// (src/ops/reduction_ops_cuda.cu:154-177), and C-ABI status codes become ctorch's exceptions.
#include "ctorch/allocator.h"
#include "ctorch/device.h"
#include "ctorch/dispatch.h"
#include "ctorch/dtype.h"
#include "ctorch/errors.h"
#include "ctorch/ops/op_keys.h"
#include "ctorch/tensor.h"

#include "cuda/device_guard.h"
#include "ops/reduction.h"

#include "b200_cast.h"
#include "ctb/ctb.h"

#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>

namespace ctorch {
namespace {

ctb_view view_of(const Tensor& t) {
    ctb_view v{};
    const auto& shape = t.shape();
    const auto& stride = t.stride();
    if (shape.size() > CTB_MAX_DIMS) {
        throw ShapeError("ctorch: CUDA backend does not support tensor rank > " +
                         std::to_string(CTB_MAX_DIMS) + " (got " + std::to_string(shape.size()) + ")");
    }
    v.data = static_cast<char*>(const_cast<void*>(t.storage().data())) +
             static_cast<std::size_t>(t.offset()) * size_of(t.dtype());
    v.dtype = static_cast<int32_t>(t.dtype());
    v.ndim = static_cast<int32_t>(shape.size());
    for (std::size_t d = 0; d < shape.size(); ++d) {
        v.shape[d] = shape[d];
        v.strides[d] = stride[d];
    }
    return v;
}

void check(int status, const char* name) {
    if (status == CTB_OK) return;
    const std::string msg = std::string("ctorch::") + name + ": " + ctb_last_error();
    switch (status) {
    case CTB_ERR_DTYPE: throw DTypeError(msg);
    case CTB_ERR_SHAPE:
    case CTB_ERR_INDEX: throw ShapeError(msg);
    case CTB_ERR_CUDA: throw DeviceError(msg);
    case CTB_ERR_ARGUMENT: throw std::invalid_argument(msg);
    default: throw Error(msg);
    }
}

// Scratch from ctorch's caching allocator for the device (returned on scope exit; every use is
// ordered on the legacy stream, so the block can be handed out again safely).
class Scratch {
  public:
    Scratch(Device d, std::size_t bytes) : device_(d), bytes_(bytes) {
        if (bytes_) ptr_ = default_allocator(d)->allocate(bytes_);
    }
    ~Scratch() {
        if (ptr_) default_allocator(device_)->deallocate(ptr_, bytes_);
    }
    Scratch(const Scratch&) = delete;
    Scratch& operator=(const Scratch&) = delete;
    void* get() const { return ptr_; }
    std::size_t size() const { return bytes_; }

  private:
    Device device_;
    std::size_t bytes_;
    void* ptr_ = nullptr;
};

constexpr ctb_stream kLegacyStream = nullptr;

// ---------------------------------------------------------------- binary

template <int OP> void binary_cuda(const Tensor& a, const Tensor& b, Tensor& out) {
    cuda::DeviceGuard guard(out.device().index);
    const ctb_view va = view_of(a), vb = view_of(b), vo = view_of(out);
    check(ctb_binary(OP, &va, &vb, &vo, kLegacyStream), OP == CTB_ADD ? "add" : OP == CTB_SUB ? "sub" : OP == CTB_MUL ? "mul" : "div");
}

template <int OP> void binary_inplace_cuda(Tensor& a, const Tensor& b) {
    cuda::DeviceGuard guard(a.device().index);
    const ctb_view va = view_of(a), vb = view_of(b);
    check(ctb_binary(OP, &va, &vb, &va, kLegacyStream), OP == CTB_ADD ? "add_" : OP == CTB_SUB ? "sub_" : OP == CTB_MUL ? "mul_" : "div_");
}

// ---------------------------------------------------------------- unary

template <int OP> void unary_cuda(const Tensor& in, Tensor& out) {
    static const char* names[] = {"neg", "abs", "exp", "log", "sqrt", "relu", "sigmoid", "tanh"};
    cuda::DeviceGuard guard(out.device().index);
    const ctb_view vi = view_of(in), vo = view_of(out);
    check(ctb_unary(OP, &vi, &vo, kLegacyStream), names[OP]);
}

// ---------------------------------------------------------------- reductions

uint32_t mask_of(const ops::ReductionAxes& ax) {
    uint32_t m = 0;
    for (int d = 0; d < ax.rank; ++d)
        if (ax.reduce[static_cast<std::size_t>(d)]) m |= 1u << d;
    return m;
}

template <int OP> void reduce_cuda(const Tensor& in, Tensor& out, const ops::ReductionAxes& ax) {
    static const char* names[] = {"sum", "mean", "prod", "max", "min"};
    cuda::DeviceGuard guard(out.device().index);
    const ctb_view vi = view_of(in), vo = view_of(out);
    const uint32_t mask = mask_of(ax);
    Scratch scratch(out.device(), ctb_reduce_scratch_bytes(OP, &vi, &vo, mask));
    check(ctb_reduce(OP, &vi, &vo, mask, scratch.get(), scratch.size(), kLegacyStream), names[OP]);
}

template <int OP> void reduce_idx_cuda(const Tensor& in, Tensor& vals, Tensor& idx, int axis) {
    cuda::DeviceGuard guard(idx.device().index);
    const ctb_view vi = view_of(in), vv = view_of(vals), vx = view_of(idx);
    Scratch scratch(idx.device(), ctb_reduce_index_scratch_bytes(&vi, axis));
    check(ctb_reduce_index(OP, &vi, &vv, &vx, axis, scratch.get(), scratch.size(), kLegacyStream),
          OP == CTB_MAX ? "max" : "min");
}

template <int OP> void arg_cuda(const Tensor& in, Tensor& idx, int axis) {
    cuda::DeviceGuard guard(idx.device().index);
    const ctb_view vi = view_of(in), vx = view_of(idx);
    Scratch scratch(idx.device(), ctb_reduce_index_scratch_bytes(&vi, axis));
    check(ctb_reduce_index(OP, &vi, nullptr, &vx, axis, scratch.get(), scratch.size(), kLegacyStream),
          OP == CTB_MAX ? "argmax" : "argmin");
}

// ---------------------------------------------------------------- index_select

void index_select_cuda(const Tensor& src, int dim, const Tensor& indices, Tensor& out) {
    cuda::DeviceGuard guard(out.device().index);
    const ctb_view vs = view_of(src), vi = view_of(indices), vo = view_of(out);
    Scratch status(out.device(), 16);
    check(ctb_index_select(&vs, dim, &vi, &vo, static_cast<int32_t*>(status.get()), kLegacyStream),
          "index_select");
    // Synchronous error report, as ctorch's CUDA path does (src/ops/indexing_cuda.cu:186-194); the
    // copy waits for the validation and gather launches on the legacy stream.
    struct {
        int32_t flag;
        int32_t pad;
        int64_t bad;
    } host{};
    if (cudaMemcpy(&host, status.get(), sizeof(host), cudaMemcpyDeviceToHost) != cudaSuccess) {
        throw DeviceError("ctorch::index_select: cudaMemcpy of the status word failed");
    }
    if (host.flag != 0) {
        throw ShapeError("ctorch::index_select: index " + std::to_string(host.bad) +
                         " out of range for dim " + std::to_string(dim) + " of size " +
                         std::to_string(src.shape()[static_cast<std::size_t>(dim)]));
    }
}

}  // namespace

// ---------------------------------------------------------------- cast / contiguous (b200_cast.h)

namespace b200 {

Tensor cast_cuda(const Tensor& t, dtype target) {
    if (!t.device().is_cuda()) throw DeviceError("ctorch::b200::cast_cuda: tensor not on a CUDA device");
    if (t.dtype() == target && t.is_contiguous() && t.offset() == 0) return t;
    Tensor out(t.shape(), target, t.device());
    cuda::DeviceGuard guard(t.device().index);
    const ctb_view vi = view_of(t), vo = view_of(out);
    check(ctb_cast(&vi, &vo, kLegacyStream), "cast");
    return out;
}

Tensor contiguous_cuda(const Tensor& t) { return cast_cuda(t, t.dtype()); }

}  // namespace b200

extern "C" void ctorch_register_cuda_binary_ops() {
    dispatch::register_op<op::AddOp>(Device::Kind::CUDA, &binary_cuda<CTB_ADD>);
    dispatch::register_op<op::SubOp>(Device::Kind::CUDA, &binary_cuda<CTB_SUB>);
    dispatch::register_op<op::MulOp>(Device::Kind::CUDA, &binary_cuda<CTB_MUL>);
    dispatch::register_op<op::DivOp>(Device::Kind::CUDA, &binary_cuda<CTB_DIV>);
    dispatch::register_op<op::AddInplaceOp>(Device::Kind::CUDA, &binary_inplace_cuda<CTB_ADD>);
    dispatch::register_op<op::SubInplaceOp>(Device::Kind::CUDA, &binary_inplace_cuda<CTB_SUB>);
    dispatch::register_op<op::MulInplaceOp>(Device::Kind::CUDA, &binary_inplace_cuda<CTB_MUL>);
    dispatch::register_op<op::DivInplaceOp>(Device::Kind::CUDA, &binary_inplace_cuda<CTB_DIV>);
}

extern "C" void ctorch_register_cuda_unary_ops() {
    dispatch::register_op<op::NegOp>(Device::Kind::CUDA, &unary_cuda<CTB_NEG>);
    dispatch::register_op<op::AbsOp>(Device::Kind::CUDA, &unary_cuda<CTB_ABS>);
    dispatch::register_op<op::ExpOp>(Device::Kind::CUDA, &unary_cuda<CTB_EXP>);
    dispatch::register_op<op::LogOp>(Device::Kind::CUDA, &unary_cuda<CTB_LOG>);
    dispatch::register_op<op::SqrtOp>(Device::Kind::CUDA, &unary_cuda<CTB_SQRT>);
    dispatch::register_op<op::ReluOp>(Device::Kind::CUDA, &unary_cuda<CTB_RELU>);
    dispatch::register_op<op::SigmoidOp>(Device::Kind::CUDA, &unary_cuda<CTB_SIGMOID>);
    dispatch::register_op<op::TanhOp>(Device::Kind::CUDA, &unary_cuda<CTB_TANH>);
}

extern "C" void ctorch_register_cuda_reduction_ops() {
    dispatch::register_op<op::SumOp>(Device::Kind::CUDA, &reduce_cuda<CTB_SUM>);
    dispatch::register_op<op::ProdOp>(Device::Kind::CUDA, &reduce_cuda<CTB_PROD>);
    dispatch::register_op<op::MeanOp>(Device::Kind::CUDA, &reduce_cuda<CTB_MEAN>);
    dispatch::register_op<op::MaxValOp>(Device::Kind::CUDA, &reduce_cuda<CTB_MAX>);
    dispatch::register_op<op::MinValOp>(Device::Kind::CUDA, &reduce_cuda<CTB_MIN>);
    dispatch::register_op<op::MaxValIdxOp>(Device::Kind::CUDA, &reduce_idx_cuda<CTB_MAX>);
    dispatch::register_op<op::MinValIdxOp>(Device::Kind::CUDA, &reduce_idx_cuda<CTB_MIN>);
    dispatch::register_op<op::ArgmaxOp>(Device::Kind::CUDA, &arg_cuda<CTB_MAX>);
    dispatch::register_op<op::ArgminOp>(Device::Kind::CUDA, &arg_cuda<CTB_MIN>);
}

extern "C" void ctorch_register_cuda_indexing_ops() {
    dispatch::register_op<op::IndexSelectOp>(Device::Kind::CUDA, &index_select_cuda);
}

}  // namespace ctorch
