/*
 * ctb_oracle.c — CPU restatement of ctorch's CPU backend (TEST INFRASTRUCTURE ONLY).
 *
 * Used by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg as the checker for the
 * CUDA backend in ctorch_b200/. It is never the thing measured on the GPU and the product never
 * links it. Citations are file:line in the ctorch source tree.
 *
 * Restated semantics, in brief:
 *   - binary ops: signed integers wrap through unsigned arithmetic (src/ops/functors.h:39-66);
 *     float ops are single IEEE operations in the output dtype; operands are first converted with
 *     static_cast semantics (src/ops/cast_cpu.cpp:21-27, bool -> 0/1).
 *   - relu propagates NaN, maps -0.0 to +0.0 (src/ops/functors.h:107-119).
 *   - reductions walk the kept subspace in row-major order and, per output, the reduced subspace
 *     in row-major order, folding sequentially into the accumulator
 *     (src/ops/reduction_ops_cpu.cpp:49-94); fp32 sum/prod/mean accumulate in double.
 *   - mean = T(sum) then *= T(1)/T(N), NaN when N == 0 (src/ops/reduction_ops_cpu.cpp:160-175).
 *   - max/min seed with +-inf / type limits and replace on a strict compare with NaN adoption
 *     (src/ops/reduction_functors.h:55-110).
 *   - max/min with index seed with element 0 and index 0 (src/ops/reduction_ops_cpu.cpp:236-297).
 *   - index_select validates every index before any gather (src/ops/indexing_cpu.cpp:35-101).
 */
#include "ctb_oracle.h"

#include <math.h>
#include <stddef.h>
#include <string.h>

/* ------------------------------------------------------------------ helpers */

static int64_t view_numel(const orc_view* v) {
    int64_t n = 1;
    for (int d = 0; d < v->ndim; ++d) n *= v->shape[d];
    return n;
}

static size_t dtype_size(int dt) {
    switch (dt) {
    case ORC_F32: return 4;
    case ORC_F64: return 8;
    case ORC_I32: return 4;
    case ORC_I64: return 8;
    case ORC_BOOL: return 1;
    case ORC_BF16: return 2;
    }
    return 0;
}

/* src/type_promotion.cpp:45-56 — the 5x5 lattice bool < int32 < int64 < float32 < float64. */
int orc_promote(int a, int b) {
    static const int rank_of[5] = {3, 4, 1, 2, 0}; /* f32, f64, i32, i64, bool */
    static const int dtype_of_rank[5] = {ORC_BOOL, ORC_I32, ORC_I64, ORC_F32, ORC_F64};
    if (a < 0 || a > 4 || b < 0 || b > 4) return -1;
    int ra = rank_of[a], rb = rank_of[b];
    return dtype_of_rank[ra > rb ? ra : rb];
}

static const char* elem_ptr(const orc_view* v, int64_t off) {
    return (const char*)v->data + off * (int64_t)dtype_size(v->dtype);
}

/* static_cast loads (src/ops/cast_cpu.cpp:21-27). */
static double ld_f64(const orc_view* v, int64_t off) {
    const char* p = elem_ptr(v, off);
    switch (v->dtype) {
    case ORC_F32: return (double)*(const float*)p;
    case ORC_F64: return *(const double*)p;
    case ORC_I32: return (double)*(const int32_t*)p;
    case ORC_I64: return (double)*(const int64_t*)p;
    case ORC_BOOL: return *(const uint8_t*)p ? 1.0 : 0.0;
    }
    return 0.0;
}
static float ld_f32(const orc_view* v, int64_t off) {
    const char* p = elem_ptr(v, off);
    switch (v->dtype) {
    case ORC_F32: return *(const float*)p;
    case ORC_F64: return (float)*(const double*)p;
    case ORC_I32: return (float)*(const int32_t*)p;
    case ORC_I64: return (float)*(const int64_t*)p;
    case ORC_BOOL: return *(const uint8_t*)p ? 1.0f : 0.0f;
    }
    return 0.0f;
}
static int64_t ld_i64(const orc_view* v, int64_t off) {
    const char* p = elem_ptr(v, off);
    switch (v->dtype) {
    case ORC_F32: return (int64_t)*(const float*)p;
    case ORC_F64: return (int64_t)*(const double*)p;
    case ORC_I32: return (int64_t)*(const int32_t*)p;
    case ORC_I64: return *(const int64_t*)p;
    case ORC_BOOL: return *(const uint8_t*)p ? 1 : 0;
    }
    return 0;
}
static int32_t ld_i32(const orc_view* v, int64_t off) {
    const char* p = elem_ptr(v, off);
    switch (v->dtype) {
    case ORC_F32: return (int32_t)*(const float*)p;
    case ORC_F64: return (int32_t)*(const double*)p;
    case ORC_I32: return *(const int32_t*)p;
    case ORC_I64: return (int32_t)*(const int64_t*)p;
    case ORC_BOOL: return *(const uint8_t*)p ? 1 : 0;
    }
    return 0;
}

/* Right-aligned broadcast of `in` to `out_ndim`/`out_shape` (src/ops/broadcast.cpp:35-82): a
 * missing or size-1 dim gets stride 0. Returns 0 if the shapes are incompatible. */
static int broadcast_strides(const orc_view* in, int out_ndim, const int64_t* out_shape,
                             int64_t* strides) {
    if (in->ndim > out_ndim) return 0;
    for (int i = 0; i < out_ndim; ++i) {
        int j = i - (out_ndim - in->ndim);
        if (j < 0) {
            strides[i] = 0;
            continue;
        }
        if (in->shape[j] == out_shape[i]) {
            strides[i] = in->shape[j] == 1 ? 0 : in->strides[j];
        } else if (in->shape[j] == 1) {
            strides[i] = 0;
        } else {
            return 0;
        }
    }
    return 1;
}

/* ---------------------------------------------------------------- binary ops */

/* src/ops/functors.h:39-66: signed integers through unsigned arithmetic; floats as-is. */
static int32_t bin_i32(int op, int32_t a, int32_t b) {
    uint32_t ua = (uint32_t)a, ub = (uint32_t)b;
    switch (op) {
    case ORC_ADD: return (int32_t)(ua + ub);
    case ORC_SUB: return (int32_t)(ua - ub);
    case ORC_MUL: return (int32_t)(ua * ub);
    }
    return 0;
}
static int64_t bin_i64(int op, int64_t a, int64_t b) {
    uint64_t ua = (uint64_t)a, ub = (uint64_t)b;
    switch (op) {
    case ORC_ADD: return (int64_t)(ua + ub);
    case ORC_SUB: return (int64_t)(ua - ub);
    case ORC_MUL: return (int64_t)(ua * ub);
    }
    return 0;
}
static float bin_f32(int op, float a, float b) {
    switch (op) {
    case ORC_ADD: return a + b;
    case ORC_SUB: return a - b;
    case ORC_MUL: return a * b;
    case ORC_DIV: return a / b;
    }
    return 0.0f;
}
static double bin_f64(int op, double a, double b) {
    switch (op) {
    case ORC_ADD: return a + b;
    case ORC_SUB: return a - b;
    case ORC_MUL: return a * b;
    case ORC_DIV: return a / b;
    }
    return 0.0;
}

/* Binary front-door + kernel: src/ops/binary_ops_cpu.cpp:43-111 (kernel, int-div refusal),
 * :202-220 (bool refusal is the front-door's job; here bool is only refused as an output dtype,
 * as binary_dispatch_numeric does at :81-83), iteration as src/ops/tensor_iter.h:84-109. */
int orc_binary(int op, const orc_view* a, const orc_view* b, const orc_view* out) {
    if (op < ORC_ADD || op > ORC_DIV) return ORC_ERR_DTYPE;
    int pt = orc_promote(a->dtype, b->dtype);
    if (pt < 0 || out->dtype != pt) return ORC_ERR_DTYPE;
    if (out->dtype == ORC_BOOL || out->dtype == ORC_BF16) return ORC_ERR_DTYPE;
    if (op == ORC_DIV && (out->dtype == ORC_I32 || out->dtype == ORC_I64)) return ORC_ERR_DTYPE;
    if (a->ndim > ORC_MAX_DIMS || b->ndim > ORC_MAX_DIMS || out->ndim > ORC_MAX_DIMS)
        return ORC_ERR_SHAPE;

    int64_t sa[ORC_MAX_DIMS], sb[ORC_MAX_DIMS];
    if (!broadcast_strides(a, out->ndim, out->shape, sa)) return ORC_ERR_SHAPE;
    if (!broadcast_strides(b, out->ndim, out->shape, sb)) return ORC_ERR_SHAPE;

    const int r = out->ndim;
    const int64_t n = view_numel(out);
    int64_t idx[ORC_MAX_DIMS] = {0};
    int64_t ao = 0, bo = 0, oo = 0;
    for (int64_t i = 0; i < n; ++i) {
        char* po = (char*)out->data + oo * (int64_t)dtype_size(out->dtype);
        switch (out->dtype) {
        case ORC_F32: *(float*)po = bin_f32(op, ld_f32(a, ao), ld_f32(b, bo)); break;
        case ORC_F64: *(double*)po = bin_f64(op, ld_f64(a, ao), ld_f64(b, bo)); break;
        case ORC_I32: *(int32_t*)po = bin_i32(op, ld_i32(a, ao), ld_i32(b, bo)); break;
        case ORC_I64: *(int64_t*)po = bin_i64(op, ld_i64(a, ao), ld_i64(b, bo)); break;
        }
        for (int d = r - 1; d >= 0; --d) {
            ++idx[d];
            ao += sa[d];
            bo += sb[d];
            oo += out->strides[d];
            if (idx[d] < out->shape[d]) break;
            idx[d] = 0;
            ao -= sa[d] * out->shape[d];
            bo -= sb[d] * out->shape[d];
            oo -= out->strides[d] * out->shape[d];
        }
    }
    return ORC_OK;
}

/* ----------------------------------------------------------------- unary ops */

/* src/ops/functors.h:70-160. */
static float un_f32(int op, float x) {
    switch (op) {
    case ORC_NEG: return -x;
    case ORC_ABS: return fabsf(x);
    case ORC_RELU: if (x != x) return x; return x > 0.0f ? x : 0.0f;
    case ORC_EXP: return expf(x);
    case ORC_LOG: return logf(x);
    case ORC_SQRT: return sqrtf(x);
    case ORC_SIGMOID: {
        if (x >= 0.0f) return 1.0f / (1.0f + expf(-x));
        float e = expf(x);
        return e / (1.0f + e);
    }
    case ORC_TANH: return tanhf(x);
    }
    return 0.0f;
}
static double un_f64(int op, double x) {
    switch (op) {
    case ORC_NEG: return -x;
    case ORC_ABS: return fabs(x);
    case ORC_RELU: if (x != x) return x; return x > 0.0 ? x : 0.0;
    case ORC_EXP: return exp(x);
    case ORC_LOG: return log(x);
    case ORC_SQRT: return sqrt(x);
    case ORC_SIGMOID: {
        if (x >= 0.0) return 1.0 / (1.0 + exp(-x));
        double e = exp(x);
        return e / (1.0 + e);
    }
    case ORC_TANH: return tanh(x);
    }
    return 0.0;
}
static int64_t un_int(int op, int64_t x, int bits) {
    /* NegF / AbsF through unsigned arithmetic (functors.h:75-104); ReluF (:117). */
    if (bits == 32) {
        int32_t v = (int32_t)x;
        switch (op) {
        case ORC_NEG: return (int32_t)(0u - (uint32_t)v);
        case ORC_ABS: return v >= 0 ? v : (int32_t)(0u - (uint32_t)v);
        case ORC_RELU: return v > 0 ? v : 0;
        }
    } else {
        switch (op) {
        case ORC_NEG: return (int64_t)(0ull - (uint64_t)x);
        case ORC_ABS: return x >= 0 ? x : (int64_t)(0ull - (uint64_t)x);
        case ORC_RELU: return x > 0 ? x : 0;
        }
    }
    return 0;
}

/* src/ops/unary_ops_cpu.cpp:37-110 (kernel + dtype dispatch; float-only transcendental ops). */
int orc_unary(int op, const orc_view* in, const orc_view* out) {
    if (op < ORC_NEG || op > ORC_TANH) return ORC_ERR_DTYPE;
    if (in->dtype != out->dtype) return ORC_ERR_DTYPE;
    if (in->ndim != out->ndim) return ORC_ERR_SHAPE;
    for (int d = 0; d < in->ndim; ++d)
        if (in->shape[d] != out->shape[d]) return ORC_ERR_SHAPE;
    const int dt = out->dtype;
    const int is_int_op = (op == ORC_NEG || op == ORC_ABS || op == ORC_RELU);
    if (dt == ORC_BOOL || dt == ORC_BF16) return ORC_ERR_DTYPE;
    if (!is_int_op && (dt == ORC_I32 || dt == ORC_I64)) return ORC_ERR_DTYPE;

    const int r = out->ndim;
    const int64_t n = view_numel(out);
    int64_t idx[ORC_MAX_DIMS] = {0};
    int64_t io = 0, oo = 0;
    const size_t es = dtype_size(dt);
    for (int64_t i = 0; i < n; ++i) {
        const char* pi = (const char*)in->data + io * (int64_t)es;
        char* po = (char*)out->data + oo * (int64_t)es;
        switch (dt) {
        case ORC_F32: *(float*)po = un_f32(op, *(const float*)pi); break;
        case ORC_F64: *(double*)po = un_f64(op, *(const double*)pi); break;
        case ORC_I32: *(int32_t*)po = (int32_t)un_int(op, *(const int32_t*)pi, 32); break;
        case ORC_I64: *(int64_t*)po = un_int(op, *(const int64_t*)pi, 64); break;
        }
        for (int d = r - 1; d >= 0; --d) {
            ++idx[d];
            io += in->strides[d];
            oo += out->strides[d];
            if (idx[d] < out->shape[d]) break;
            idx[d] = 0;
            io -= in->strides[d] * out->shape[d];
            oo -= out->strides[d] * out->shape[d];
        }
    }
    return ORC_OK;
}

/* ---------------------------------------------------------------------- cast */

/* src/ops/cast_cpu.cpp:21-90: out = static_cast<out dtype>(in) elementwise over the same shape,
 * bool read as 0/1 (the static_cast loads above) and written as (value != 0). */
int orc_cast(const orc_view* in, const orc_view* out) {
    if (in->dtype == ORC_BF16 || out->dtype == ORC_BF16) return ORC_ERR_DTYPE;
    if (in->ndim != out->ndim) return ORC_ERR_SHAPE;
    for (int d = 0; d < in->ndim; ++d)
        if (in->shape[d] != out->shape[d]) return ORC_ERR_SHAPE;
    const int r = out->ndim;
    const int64_t n = view_numel(out);
    int64_t idx[ORC_MAX_DIMS] = {0};
    int64_t io = 0, oo = 0;
    const size_t es = dtype_size(out->dtype);
    for (int64_t i = 0; i < n; ++i) {
        char* po = (char*)out->data + oo * (int64_t)es;
        switch (out->dtype) {
        case ORC_F32: *(float*)po = ld_f32(in, io); break;
        case ORC_F64: *(double*)po = ld_f64(in, io); break;
        case ORC_I32: *(int32_t*)po = ld_i32(in, io); break;
        case ORC_I64: *(int64_t*)po = ld_i64(in, io); break;
        case ORC_BOOL: {
            const char* pi = elem_ptr(in, io);
            int nz = 0;
            switch (in->dtype) {
            case ORC_F32: nz = *(const float*)pi != 0.0f; break;
            case ORC_F64: nz = *(const double*)pi != 0.0; break;
            case ORC_I32: nz = *(const int32_t*)pi != 0; break;
            case ORC_I64: nz = *(const int64_t*)pi != 0; break;
            case ORC_BOOL: nz = *(const uint8_t*)pi != 0; break;
            }
            *(uint8_t*)po = (uint8_t)nz;
            break;
        }
        }
        for (int d = r - 1; d >= 0; --d) {
            ++idx[d];
            io += in->strides[d];
            oo += out->strides[d];
            if (idx[d] < out->shape[d]) break;
            idx[d] = 0;
            io -= in->strides[d] * out->shape[d];
            oo -= out->strides[d] * out->shape[d];
        }
    }
    return ORC_OK;
}

/* ---------------------------------------------------------------- reductions */

typedef struct {
    int rank_kept, rank_red;
    int64_t shape_kept[ORC_MAX_DIMS], shape_red[ORC_MAX_DIMS];
    int64_t stride_kept[ORC_MAX_DIMS], stride_red[ORC_MAX_DIMS];
    int64_t stride_out[ORC_MAX_DIMS];
    int64_t kept_numel, red_numel;
} red_plan;

/* src/ops/reduction_iter.cpp:20-69 — split shape/stride into kept and reduced halves; output dim
 * cursor advances on every input dim with keepdim (out rank == in rank), else on kept dims only. */
static int make_plan(const orc_view* in, const orc_view* out, uint32_t mask, red_plan* p) {
    memset(p, 0, sizeof(*p));
    p->kept_numel = 1;
    p->red_numel = 1;
    int n_kept = 0;
    for (int d = 0; d < in->ndim; ++d)
        if (!((mask >> d) & 1u)) ++n_kept;
    const int keepdim = (out->ndim == in->ndim);
    if (!keepdim && out->ndim != n_kept) return ORC_ERR_SHAPE;
    int od = 0;
    for (int d = 0; d < in->ndim; ++d) {
        const int red = (mask >> d) & 1u;
        if (red) {
            p->shape_red[p->rank_red] = in->shape[d];
            p->stride_red[p->rank_red] = in->strides[d];
            p->red_numel *= in->shape[d];
            ++p->rank_red;
            if (keepdim && out->shape[od] != 1) return ORC_ERR_SHAPE;
        } else {
            if (out->shape[od] != in->shape[d]) return ORC_ERR_SHAPE;
            p->shape_kept[p->rank_kept] = in->shape[d];
            p->stride_kept[p->rank_kept] = in->strides[d];
            p->stride_out[p->rank_kept] = out->strides[od];
            p->kept_numel *= in->shape[d];
            ++p->rank_kept;
        }
        if (keepdim || !red) ++od;
    }
    return ORC_OK;
}

/* MaxF / MinF::should_replace (src/ops/reduction_functors.h:73-83, :99-109). */
static int repl_f(int is_max, double cur, double v) {
    if (cur != cur) return 0;
    if (v != v) return 1;
    return is_max ? v > cur : v < cur;
}
static int repl_i(int is_max, int64_t cur, int64_t v) { return is_max ? v > cur : v < cur; }

/* src/ops/reduction_ops_cpu.cpp:49-94 (run_reduction), :98-175 (sum/prod/mean dtype dispatch),
 * :199-229 (values-only max/min); dtype rules src/ops/reduction.cpp:131-153. */
int orc_reduce(int op, const orc_view* in, const orc_view* out, uint32_t mask) {
    if (op < ORC_SUM || op > ORC_MIN) return ORC_ERR_DTYPE;
    const int dt = in->dtype;
    if (dt == ORC_BF16 || dt < 0 || dt > ORC_BOOL) return ORC_ERR_DTYPE;
    if (in->ndim > ORC_MAX_DIMS) return ORC_ERR_SHAPE;
    if (in->ndim < 32 && (mask >> in->ndim) != 0u) return ORC_ERR_SHAPE;
    const int is_float = (dt == ORC_F32 || dt == ORC_F64);
    int want_out;
    if (op == ORC_SUM || op == ORC_PROD) want_out = is_float ? dt : ORC_I64;
    else if (op == ORC_MEAN) {
        if (!is_float) return ORC_ERR_DTYPE;
        want_out = dt;
    } else want_out = dt;
    if (out->dtype != want_out) return ORC_ERR_DTYPE;

    red_plan p;
    int st = make_plan(in, out, mask, &p);
    if (st != ORC_OK) return st;

    const size_t os = dtype_size(out->dtype);
    int64_t kidx[ORC_MAX_DIMS] = {0};
    int64_t in_kept = 0, out_off = 0;
    for (int64_t k = 0; k < p.kept_numel; ++k) {
        int64_t ridx[ORC_MAX_DIMS] = {0};
        int64_t in_red = 0;
        /* Accumulators: double for float sum/prod/mean; uint64 (two's-complement wrap) for integer
         * sum/prod; T for max/min. */
        double accd = 0.0;
        uint64_t accu = 0;
        int64_t acci = 0;
        float accf = 0.0f;
        const int is_max = (op == ORC_MAX);
        if (op == ORC_SUM || op == ORC_MEAN) { accd = 0.0; accu = 0; }
        else if (op == ORC_PROD) { accd = 1.0; accu = 1; }
        else {
            switch (dt) {
            case ORC_F32: accf = is_max ? -INFINITY : INFINITY; break;
            case ORC_F64: accd = is_max ? -INFINITY : INFINITY; break;
            case ORC_I32: acci = is_max ? INT32_MIN : INT32_MAX; break;
            case ORC_I64: acci = is_max ? INT64_MIN : INT64_MAX; break;
            case ORC_BOOL: acci = is_max ? 0 : 255; break;
            }
        }
        for (int64_t r = 0; r < p.red_numel; ++r) {
            const int64_t off = in_kept + in_red;
            if (op == ORC_SUM || op == ORC_MEAN || op == ORC_PROD) {
                if (is_float) {
                    const double v = ld_f64(in, off);
                    if (op == ORC_PROD) accd *= v; else accd += v;
                } else {
                    const uint64_t v = (uint64_t)ld_i64(in, off);
                    if (op == ORC_PROD) accu *= v; else accu += v;
                }
            } else {
                switch (dt) {
                case ORC_F32: {
                    const float v = ld_f32(in, off);
                    if (repl_f(is_max, accf, v)) accf = v;
                    break;
                }
                case ORC_F64: {
                    const double v = ld_f64(in, off);
                    if (repl_f(is_max, accd, v)) accd = v;
                    break;
                }
                default: {
                    const int64_t v = ld_i64(in, off);
                    if (repl_i(is_max, acci, v)) acci = v;
                    break;
                }
                }
            }
            for (int d = p.rank_red - 1; d >= 0; --d) {
                ++ridx[d];
                in_red += p.stride_red[d];
                if (ridx[d] < p.shape_red[d]) break;
                ridx[d] = 0;
                in_red -= p.stride_red[d] * p.shape_red[d];
            }
        }
        char* po = (char*)out->data + out_off * (int64_t)os;
        if (op == ORC_SUM || op == ORC_PROD) {
            if (dt == ORC_F32) *(float*)po = (float)accd;
            else if (dt == ORC_F64) *(double*)po = accd;
            else *(int64_t*)po = (int64_t)accu;
        } else if (op == ORC_MEAN) {
            if (dt == ORC_F32) {
                float s = (float)accd;
                if (p.red_numel == 0) s = NAN;
                else s *= 1.0f / (float)p.red_numel;
                *(float*)po = s;
            } else {
                double s = accd;
                if (p.red_numel == 0) s = NAN;
                else s *= 1.0 / (double)p.red_numel;
                *(double*)po = s;
            }
        } else {
            switch (dt) {
            case ORC_F32: *(float*)po = accf; break;
            case ORC_F64: *(double*)po = accd; break;
            case ORC_I32: *(int32_t*)po = (int32_t)acci; break;
            case ORC_I64: *(int64_t*)po = acci; break;
            case ORC_BOOL: *(uint8_t*)po = (uint8_t)acci; break;
            }
        }
        for (int d = p.rank_kept - 1; d >= 0; --d) {
            ++kidx[d];
            in_kept += p.stride_kept[d];
            out_off += p.stride_out[d];
            if (kidx[d] < p.shape_kept[d]) break;
            kidx[d] = 0;
            in_kept -= p.stride_kept[d] * p.shape_kept[d];
            out_off -= p.stride_out[d] * p.shape_kept[d];
        }
    }
    return ORC_OK;
}

/* src/ops/reduction_ops_cpu.cpp:236-297 (run_axis_with_idx_cpu): seed with element 0 / index 0,
 * replace on should_replace. A zero-length axis is refused (the front-door throws ShapeError,
 * reduction_ops_cpu.cpp:433-436). */
int orc_reduce_idx(int op, const orc_view* in, const orc_view* vals, const orc_view* idx,
                   int axis) {
    if (op != ORC_MAX && op != ORC_MIN) return ORC_ERR_DTYPE;
    const int dt = in->dtype;
    if (dt == ORC_BF16 || dt < 0 || dt > ORC_BOOL) return ORC_ERR_DTYPE;
    if (idx->dtype != ORC_I64) return ORC_ERR_DTYPE;
    if (vals && vals->dtype != dt) return ORC_ERR_DTYPE;
    if (axis < 0 || axis >= in->ndim) return ORC_ERR_SHAPE;
    if (in->shape[axis] == 0) return ORC_ERR_SHAPE;
    red_plan pi, pv;
    int st = make_plan(in, idx, 1u << axis, &pi);
    if (st != ORC_OK) return st;
    if (vals) {
        st = make_plan(in, vals, 1u << axis, &pv);
        if (st != ORC_OK) return st;
    }
    const int is_max = (op == ORC_MAX);
    const int64_t rsize = in->shape[axis], rstride = in->strides[axis];
    const size_t es = dtype_size(dt);
    int64_t kidx[ORC_MAX_DIMS] = {0};
    int64_t in_kept = 0, io = 0, vo = 0;
    for (int64_t k = 0; k < pi.kept_numel; ++k) {
        int64_t best_idx = 0;
        if (dt == ORC_F32 || dt == ORC_F64) {
            double best = ld_f64(in, in_kept); /* exact for f32 as well */
            for (int64_t r = 1; r < rsize; ++r) {
                const double v = ld_f64(in, in_kept + r * rstride);
                if (repl_f(is_max, best, v)) { best = v; best_idx = r; }
            }
        } else {
            int64_t best = ld_i64(in, in_kept);
            for (int64_t r = 1; r < rsize; ++r) {
                const int64_t v = ld_i64(in, in_kept + r * rstride);
                if (repl_i(is_max, best, v)) { best = v; best_idx = r; }
            }
        }
        if (vals) {
            /* Copy the winning element's bytes (keeps NaN payloads and the sign of zero). */
            memcpy((char*)vals->data + vo * (int64_t)es, elem_ptr(in, in_kept + best_idx * rstride),
                   es);
        }
        *((int64_t*)idx->data + io) = best_idx;
        for (int d = pi.rank_kept - 1; d >= 0; --d) {
            ++kidx[d];
            in_kept += pi.stride_kept[d];
            io += pi.stride_out[d];
            if (vals) vo += pv.stride_out[d];
            if (kidx[d] < pi.shape_kept[d]) break;
            kidx[d] = 0;
            in_kept -= pi.stride_kept[d] * pi.shape_kept[d];
            io -= pi.stride_out[d] * pi.shape_kept[d];
            if (vals) vo -= pv.stride_out[d] * pi.shape_kept[d];
        }
    }
    return ORC_OK;
}

/* ------------------------------------------------------------- index_select */

/* src/ops/indexing_cpu.cpp:35-101: validate + normalise every index first (range check before
 * adding the axis size, so INT64_MIN is caught), then walk the output as an odometer with the
 * dim-th coordinate replaced by the resolved index. */
int orc_index_select(const orc_view* src, int dim, const orc_view* idx, const orc_view* out,
                     int64_t* bad_index) {
    if (src->dtype == ORC_BF16 || src->dtype < 0 || src->dtype > ORC_BOOL) return ORC_ERR_DTYPE;
    if (idx->dtype != ORC_I32 && idx->dtype != ORC_I64) return ORC_ERR_DTYPE;
    if (out->dtype != src->dtype) return ORC_ERR_DTYPE;
    if (idx->ndim != 1) return ORC_ERR_SHAPE;
    if (src->ndim == 0 || dim < 0 || dim >= src->ndim) return ORC_ERR_SHAPE;
    if (out->ndim != src->ndim) return ORC_ERR_SHAPE;
    for (int d = 0; d < src->ndim; ++d) {
        const int64_t want = d == dim ? idx->shape[0] : src->shape[d];
        if (out->shape[d] != want) return ORC_ERR_SHAPE;
    }
    const int64_t n_idx = idx->shape[0];
    const int64_t size = src->shape[dim];
    for (int64_t i = 0; i < n_idx; ++i) {
        const int64_t raw = ld_i64(idx, i * idx->strides[0]);
        if (raw < -size || raw >= size) {
            if (bad_index) *bad_index = raw;
            return ORC_ERR_INDEX;
        }
    }
    const int r = src->ndim;
    const int64_t total = view_numel(out);
    const size_t es = dtype_size(src->dtype);
    int64_t c[ORC_MAX_DIMS] = {0};
    for (int64_t lin = 0; lin < total; ++lin) {
        int64_t so = 0, oo = 0;
        for (int d = 0; d < r; ++d) {
            if (d == dim) {
                int64_t v = ld_i64(idx, c[d] * idx->strides[0]);
                if (v < 0) v += size;
                so += v * src->strides[d];
            } else {
                so += c[d] * src->strides[d];
            }
            oo += c[d] * out->strides[d];
        }
        memcpy((char*)out->data + oo * (int64_t)es, (const char*)src->data + so * (int64_t)es, es);
        for (int d = r - 1; d >= 0; --d) {
            if (++c[d] < out->shape[d]) break;
            c[d] = 0;
        }
    }
    return ORC_OK;
}
