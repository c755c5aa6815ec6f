/*
 * ctb_oracle.h — CPU restatement of ctorch's CPU backend for the eager
 * tensor-op hot path. TEST INFRASTRUCTURE ONLY: the tests, the smoke check
 * and bench.py's CPU-baseline leg use it as the checker. Nothing in the
 * ctorch_b200 product links, loads or calls it.
 *
 * Every function states the ctorch file:line whose behaviour it restates
 * (paths relative to the ctorch source tree). The restatement is pinned two
 * ways (see tests/test_oracle_*.py): against ctorch's own golden .npy
 * fixtures (tests/parity/fixtures, repacked into tests/golden/) and
 * bit-for-bit against ctorch's CPU backend compiled from its sources into
 * oracle/_ref/ (oracle/Makefile, target `ref`).
 */
#ifndef CTB_ORACLE_H
#define CTB_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_MAX_DIMS 16

/* dtype codes follow the enumerator order of ctorch::dtype (include/ctorch/dtype.h:24-31). */
enum { ORC_F32 = 0, ORC_F64 = 1, ORC_I32 = 2, ORC_I64 = 3, ORC_BOOL = 4, ORC_BF16 = 5 };

/* Status codes. */
enum { ORC_OK = 0, ORC_ERR_DTYPE = 1, ORC_ERR_SHAPE = 2, ORC_ERR_INDEX = 3 };

/* Binary op codes (include/ctorch/ops/op_keys.h:35-46). */
enum { ORC_ADD = 0, ORC_SUB = 1, ORC_MUL = 2, ORC_DIV = 3 };
/* Unary op codes (include/ctorch/ops/op_keys.h:69-92). */
enum { ORC_NEG = 0, ORC_ABS = 1, ORC_EXP = 2, ORC_LOG = 3, ORC_SQRT = 4, ORC_RELU = 5,
       ORC_SIGMOID = 6, ORC_TANH = 7 };
/* Reduction op codes (include/ctorch/ops/op_keys.h:109-123). */
enum { ORC_SUM = 0, ORC_MEAN = 1, ORC_PROD = 2, ORC_MAX = 3, ORC_MIN = 4 };

/* A strided host view: `data` points at element (0,...,0); strides are in elements. */
typedef struct {
    void* data;
    int32_t dtype;
    int32_t ndim;
    int64_t shape[ORC_MAX_DIMS];
    int64_t strides[ORC_MAX_DIMS];
} orc_view;

/* out = op(a, b) with right-aligned broadcasting of a and b to out's shape; each operand element
 * is converted to out's dtype first (the front-door's promote+cast), then the functor runs in that
 * dtype. out's dtype must equal promote_types(a, b). */
int orc_binary(int op, const orc_view* a, const orc_view* b, const orc_view* out);

/* out = op(in), same shape and dtype. */
int orc_unary(int op, const orc_view* in, const orc_view* out);

/* out = in converted to out's dtype (same shape, any strides). */
int orc_cast(const orc_view* in, const orc_view* out);

/* Multi-axis reduction: bit d of reduce_mask marks input dim d as reduced. out has either the
 * keepdim shape (rank == in rank) or the kept dims only. */
int orc_reduce(int op, const orc_view* in, const orc_view* out, uint32_t reduce_mask);

/* Single-axis max/min with index (op = ORC_MAX / ORC_MIN). vals may be NULL (argmax/argmin). */
int orc_reduce_idx(int op, const orc_view* in, const orc_view* vals, const orc_view* idx, int axis);

/* Gather along `dim` (already normalised). idx is 1-D int32/int64. Returns ORC_ERR_INDEX and
 * writes nothing when any index is out of range; *bad_index receives the first offender. */
int orc_index_select(const orc_view* src, int dim, const orc_view* idx, const orc_view* out,
                     int64_t* bad_index);

/* Type-promotion lattice (src/type_promotion.cpp:45-62); -1 for bfloat16 / unknown. */
int orc_promote(int a, int b);

#ifdef __cplusplus
}
#endif

#endif /* CTB_ORACLE_H */
