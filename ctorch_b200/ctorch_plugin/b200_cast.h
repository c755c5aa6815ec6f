// b200_cast.h — device-side dtype cast and strided -> contiguous copy for ctorch CUDA tensors,
// exported by the B200 backend (cuda_backend.cpp) for the two places where ctorch still routes
// CUDA data through the host:
//   * ctorch::maybe_cast (src/ops/binary_ops_cpu.cpp:154-184) copies a CUDA operand to the host,
//     casts it there and copies it back, and refuses non-contiguous operands; its comment asks
//     for "a bespoke ops::cast_cuda kernel". cast_cuda is that kernel;
//   * Tensor::contiguous() (src/tensor.cpp:239-254) materialises strided views on the CPU only;
//     contiguous_cuda does it on the device.
// Same results as ctorch's CPU cast (src/ops/cast_cpu.cpp:21-90) on every well-defined value.
#pragma once

#include "ctorch/dtype.h"
#include "ctorch/tensor.h"

namespace ctorch::b200 {

// A new contiguous CUDA tensor holding t converted to `target` (t itself if the dtype matches and
// t is contiguous from offset 0). Throws DTypeError for bfloat16, DeviceError for a CPU tensor.
Tensor cast_cuda(const Tensor& t, dtype target);

// A contiguous copy of a strided CUDA tensor (t itself if already contiguous from offset 0).
Tensor contiguous_cuda(const Tensor& t);

}  // namespace ctorch::b200
