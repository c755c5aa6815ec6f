// ref_capi.cpp — a flat C handle API over ctorch's own CPU backend, compiled from the ctorch
// sources in place (oracle/Makefile, target `ref`, output oracle/_ref/libctorch_ref.so).
//
// TEST INFRASTRUCTURE ONLY. The tests use it to pin the C restatement (ctb_oracle.c) bit-for-bit
// against ctorch itself, and bench.py's reference arm / CPU-baseline leg time ctorch's public
// front-doors through it. Every op goes through the public free functions declared in
// include/ctorch/ops/{elementwise,reduction,indexing}.h, i.e. ctorch's stock CPU code path; the
// one exception is ref_cast, ctorch's internal cast helper (no public front-door casts).
#include "ctorch/errors.h"
#include "ctorch/ops/elementwise.h"
#include "ctorch/ops/indexing.h"
#include "ctorch/ops/reduction.h"
#include "ctorch/tensor.h"
#include "ops/cast_cpu.h"

#include <cstdint>
#include <cstring>
#include <exception>
#include <string>
#include <vector>

namespace {

thread_local std::string g_last_error;

enum { REF_OK = 0, REF_ERR_DTYPE = 1, REF_ERR_SHAPE = 2, REF_ERR_DEVICE = 3, REF_ERR_ALIAS = 4,
       REF_ERR_OTHER = 9 };

ctorch::Tensor* box(ctorch::Tensor t) { return new ctorch::Tensor(std::move(t)); }
ctorch::Tensor& un(void* h) { return *static_cast<ctorch::Tensor*>(h); }

template <class F> void* guarded(int* err, F&& f) {
    try {
        void* r = f();
        if (err) *err = REF_OK;
        return r;
    } catch (const ctorch::DTypeError& e) {
        g_last_error = e.what();
        if (err) *err = REF_ERR_DTYPE;
    } catch (const ctorch::ShapeError& e) {
        g_last_error = e.what();
        if (err) *err = REF_ERR_SHAPE;
    } catch (const ctorch::DeviceError& e) {
        g_last_error = e.what();
        if (err) *err = REF_ERR_DEVICE;
    } catch (const ctorch::AliasError& e) {
        g_last_error = e.what();
        if (err) *err = REF_ERR_ALIAS;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        if (err) *err = REF_ERR_OTHER;
    }
    return nullptr;
}

} // namespace

extern "C" {

const char* ref_last_error() { return g_last_error.c_str(); }

// Contiguous CPU tensor holding a copy of `data` (nbytes = numel * size_of(dtype)).
void* ref_tensor_from(int dt, int ndim, const int64_t* shape, const void* data, int* err) {
    return guarded(err, [&]() -> void* {
        std::vector<std::int64_t> s(shape, shape + ndim);
        ctorch::Tensor t(s, static_cast<ctorch::dtype>(dt), ctorch::Device::cpu());
        const std::size_t nbytes =
            static_cast<std::size_t>(t.numel()) * ctorch::size_of(t.dtype());
        if (nbytes) std::memcpy(t.storage().data(), data, nbytes);
        return box(std::move(t));
    });
}

void ref_free(void* h) { delete static_cast<ctorch::Tensor*>(h); }

int ref_ndim(void* h) { return static_cast<int>(un(h).shape().size()); }
int ref_dtype(void* h) { return static_cast<int>(un(h).dtype()); }
void ref_shape(void* h, int64_t* out) {
    const auto& s = un(h).shape();
    for (std::size_t i = 0; i < s.size(); ++i) out[i] = s[i];
}
void ref_strides(void* h, int64_t* out) {
    const auto& s = un(h).stride();
    for (std::size_t i = 0; i < s.size(); ++i) out[i] = s[i];
}
int64_t ref_offset(void* h) { return un(h).offset(); }

// Row-major copy of the (possibly strided) tensor into `out`.
int ref_read(void* h, void* out) {
    int err = 0;
    guarded(&err, [&]() -> void* {
        ctorch::Tensor c = un(h).contiguous();
        const std::size_t es = ctorch::size_of(c.dtype());
        const std::size_t nbytes = static_cast<std::size_t>(c.numel()) * es;
        if (nbytes)
            std::memcpy(out,
                        static_cast<const char*>(c.storage().data()) +
                            static_cast<std::size_t>(c.offset()) * es,
                        nbytes);
        return nullptr;
    });
    return err;
}

// View ops (src/tensor.cpp:206-389).
void* ref_permute(void* h, int n, const int64_t* dims, int* err) {
    return guarded(err, [&]() -> void* {
        return box(un(h).permute(std::vector<std::int64_t>(dims, dims + n)));
    });
}
void* ref_slice(void* h, int dim, int64_t start, int64_t end, int64_t step, int* err) {
    return guarded(err, [&]() -> void* { return box(un(h).slice(dim, start, end, step)); });
}
void* ref_select(void* h, int dim, int64_t index, int* err) {
    return guarded(err, [&]() -> void* { return box(un(h).select(dim, index)); });
}
void* ref_reshape(void* h, int n, const int64_t* shape, int* err) {
    return guarded(err, [&]() -> void* {
        return box(un(h).reshape(std::vector<std::int64_t>(shape, shape + n)));
    });
}

// ctorch's dtype cast (src/ops/cast_cpu.cpp:62-90), the one its CUDA promotion round trip runs
// (src/ops/binary_ops_cpu.cpp:154-184). It is an in-library helper, not a public front-door.
void* ref_cast(void* h, int dt, int* err) {
    return guarded(err, [&]() -> void* {
        return box(ctorch::ops::cast_cpu(un(h), static_cast<ctorch::dtype>(dt)));
    });
}

// Binary front-doors (src/ops/binary_ops_cpu.cpp:251-254): op 0..3 = add, sub, mul, div.
void* ref_binary(int op, void* a, void* b, int* err) {
    return guarded(err, [&]() -> void* {
        switch (op) {
        case 0: return box(ctorch::add(un(a), un(b)));
        case 1: return box(ctorch::sub(un(a), un(b)));
        case 2: return box(ctorch::mul(un(a), un(b)));
        case 3: return box(ctorch::div(un(a), un(b)));
        }
        throw std::invalid_argument("ref_binary: bad op");
    });
}

// In-place front-doors (src/ops/binary_ops_cpu.cpp:256-267). Returns `a` (not a new handle).
int ref_binary_inplace(int op, void* a, void* b) {
    int err = 0;
    guarded(&err, [&]() -> void* {
        switch (op) {
        case 0: ctorch::add_(un(a), un(b)); break;
        case 1: ctorch::sub_(un(a), un(b)); break;
        case 2: ctorch::mul_(un(a), un(b)); break;
        case 3: ctorch::div_(un(a), un(b)); break;
        default: throw std::invalid_argument("ref_binary_inplace: bad op");
        }
        return nullptr;
    });
    return err;
}

// Unary front-doors (src/ops/unary_ops_cpu.cpp:160-167): neg, abs, exp, log, sqrt, relu,
// sigmoid, tanh.
void* ref_unary(int op, void* a, int* err) {
    return guarded(err, [&]() -> void* {
        switch (op) {
        case 0: return box(ctorch::neg(un(a)));
        case 1: return box(ctorch::abs(un(a)));
        case 2: return box(ctorch::exp(un(a)));
        case 3: return box(ctorch::log(un(a)));
        case 4: return box(ctorch::sqrt(un(a)));
        case 5: return box(ctorch::relu(un(a)));
        case 6: return box(ctorch::sigmoid(un(a)));
        case 7: return box(ctorch::tanh(un(a)));
        }
        throw std::invalid_argument("ref_unary: bad op");
    });
}

// Reduction front-doors (src/ops/reduction_ops_cpu.cpp:463-499): op 0..4 = sum, mean, prod,
// max, min. ndims < 0 selects the whole-tensor overload.
void* ref_reduce(int op, void* a, int ndims, const int64_t* dims, int keepdim, int* err) {
    return guarded(err, [&]() -> void* {
        const ctorch::Tensor& x = un(a);
        if (ndims < 0) {
            switch (op) {
            case 0: return box(ctorch::sum(x));
            case 1: return box(ctorch::mean(x));
            case 2: return box(ctorch::prod(x));
            case 3: return box(ctorch::max(x));
            case 4: return box(ctorch::min(x));
            }
        } else {
            std::vector<std::int64_t> d(dims, dims + ndims);
            const bool kd = keepdim != 0;
            switch (op) {
            case 0: return box(ctorch::sum(x, d, kd));
            case 1: return box(ctorch::mean(x, d, kd));
            case 2: return box(ctorch::prod(x, d, kd));
            case 3: return box(ctorch::max(x, d, kd));
            case 4: return box(ctorch::min(x, d, kd));
            }
        }
        throw std::invalid_argument("ref_reduce: bad op");
    });
}

// max/min along one dim with indices (reduction_ops_cpu.cpp:483-495): op 3 = max, 4 = min.
void* ref_reduce_idx(int op, void* a, int64_t dim, int keepdim, void** idx_out, int* err) {
    return guarded(err, [&]() -> void* {
        ctorch::ValuesIndices vi = op == 3 ? ctorch::max(un(a), dim, keepdim != 0)
                                           : ctorch::min(un(a), dim, keepdim != 0);
        *idx_out = box(std::move(vi.indices));
        return box(std::move(vi.values));
    });
}

// argmax / argmin (reduction_ops_cpu.cpp:493-498): op 3 = argmax, 4 = argmin.
void* ref_arg(int op, void* a, int64_t dim, int keepdim, int* err) {
    return guarded(err, [&]() -> void* {
        return box(op == 3 ? ctorch::argmax(un(a), dim, keepdim != 0)
                           : ctorch::argmin(un(a), dim, keepdim != 0));
    });
}

// index_select front-door (src/ops/indexing_cpu.cpp:163-200).
void* ref_index_select(void* src, int dim, void* idx, int* err) {
    return guarded(err, [&]() -> void* { return box(ctorch::index_select(un(src), dim, un(idx))); });
}

} // extern "C"
