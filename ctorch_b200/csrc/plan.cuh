// plan.cuh — host-side iteration planning: broadcast, dim collapse, and the choice between the
// vectorised, row, tiled-transpose and general kernels. Replaces ctorch's BinaryIndexer /
// ReductionPlan construction (src/ops/tensor_iter.cpp:41-84, src/ops/reduction_iter.cpp:20-69)
// for the CUDA side: instead of handing a rank-16 odometer to every thread, the planner collapses
// the iteration space first and picks a kernel shaped for what is left.
#pragma once

#include <cuda.h>  // CUtensorMap (a plain struct; the encoder is fetched from the driver at run time)

#include "common.cuh"

namespace ctb {

// Elementwise iteration space over up to 4 operands (0 = out, 1..3 = inputs).
constexpr int kMaxOps = 4;

enum class EwPath : int { Empty = 0, Flat = 1, RowsLong = 2, RowsShort = 3, Tiled = 4, General = 5, RowsMid = 6 };

// Row tiles (16-byte packs): RowsLong CTAs of 256 threads take 4 packs a thread along a row (8 on
// rows of 2048 packs or more); RowsMid warps take kRowsMidUnroll packs a lane. Rows of at least
// kRowsLongPacks go to RowsLong, rows of at least one warp tile to RowsMid, shorter ones to
// RowsShort.
constexpr int kRowsMidUnroll = 4;
constexpr int64_t kRowsLongPacks = 1024;
constexpr int64_t kRowsMidPacks = 32 * kRowsMidUnroll;

struct EwSpace {
    int nops = 0;  // out + inputs
    int rank = 0;
    int64_t shape[kMaxDims] = {};
    int64_t stride[kMaxOps][kMaxDims] = {};
    int64_t numel() const {
        int64_t n = 1;
        for (int d = 0; d < rank; ++d) n *= shape[d];
        return n;
    }
};

// Right-aligned broadcast of `v` to (rank, shape): size-1 and missing dims get stride 0
// (src/ops/broadcast.cpp:35-82). Returns false if the shapes do not broadcast.
bool broadcast_strides(const ctb_view& v, int rank, const int64_t* shape, int64_t* strides);

// Drops size-1 dims and merges adjacent dims whose strides chain for every operand
// (stride[d] == stride[d+1] * shape[d+1]). Keeps the order of out's dims. A 0-d space becomes
// rank 1 with shape [1].
void collapse(EwSpace& s);

// Kernel parameters shared by the elementwise kernels (passed by value, lives in the constant
// bank). Dims are stored outermost-first, as in ctorch.
struct EwArgs {
    void* out;
    const void* in[3];
    int rank;
    int xop;                       // Tiled: which input (1..3) is read transposed
    int pdim;                      // Tiled: the dim on which that input has stride 1
    int tiled_vec;                 // Tiled: 4-element packs are aligned (ew_tiled4)
    int64_t n;                     // total elements
    int64_t L;                     // innermost extent
    int64_t rows;                  // n / L
    int64_t vpr;                   // vectors per row (RowsLong/RowsMid/RowsShort)
    int64_t shape[kMaxDims];
    int64_t stride[kMaxOps][kMaxDims];
    FastDiv div[kMaxDims];         // divisors = shape[d]
    FastDiv aux;                   // RowsLong (set by the launcher)/RowsMid: tiles per row; RowsShort: vectors per row;
                                   // Tiled: tiles along L
    FastDiv aux2;                  // Tiled: tiles along P
};

struct EwPlan {
    EwPath path = EwPath::Empty;
    int vec = 1;
    EwSpace space;
    EwArgs args;
};

// Plans out = f(in...) given the operand views (already validated for dtype). `vec` is the number
// of elements one 16-byte pack holds for the narrowest participating type.
int plan_elementwise(const ctb_view* out, const ctb_view* const* ins, int nin, const int* sizes,
                     int vec, EwPlan& plan);

const char* ew_path_name(EwPath p);

// ------------------------------------------------------------------------------------------------
// Reductions: a kept space (one output each) and a reduced space, both collapsed.

enum class RedPath : int { Empty = 0, Inner = 1, Outer = 2, General = 3 };

struct RedSpace {
    int rank_k = 0, rank_r = 0;
    int64_t shape_k[kMaxDims] = {}, stride_k[kMaxDims] = {}, stride_o[kMaxDims] = {};
    int64_t stride_o2[kMaxDims] = {};  // second output (indices) for the with-index reductions
    int64_t shape_r[kMaxDims] = {}, stride_r[kMaxDims] = {};
    int64_t kept = 1, red = 1;
};

struct RedArgs {
    const void* in;
    void* out;   // values (or sum/mean/prod result)
    void* out2;  // indices (with-index reductions)
    void* scratch;
    int rank_k, rank_r;
    int split;          // S: CTAs that share one output's reduced range (1 = no combine pass)
    int64_t kept, red;  // numels
    int64_t chunk;      // reduced elements per split
    int64_t N;          // Outer: contiguous kept extent
    int64_t K;          // Outer: reduced extent; Inner: row length
    int64_t strideK;    // Outer: stride of the reduced dim
    int64_t shape_k[kMaxDims], stride_k[kMaxDims], stride_o[kMaxDims], stride_o2[kMaxDims];
    int64_t shape_r[kMaxDims], stride_r[kMaxDims];
    FastDiv div_k[kMaxDims];
    FastDiv div_r[kMaxDims];
    FastDiv aux;        // Outer: column tiles; Inner: splits
    FastDiv aux2;       // Outer: splits (bulk column kernel: the reduced extent K)
    // Bulk column kernel: CTA c folds the row-steps [c*sk_q + min(c, sk_r), ...) of the
    // flattened (column tile, row) space, sk_q or sk_q + 1 of them. CTA c's partial for tile s
    // (when it shares s with other CTAs) is partial row c + s of the scratch.
    int64_t sk_q, sk_r;
    // Strip column kernel: each batch row's N columns are cut into `aux` strips of at most
    // strip_pk 16-byte packs; unit u = (batch row u / aux, strip u % aux); CTA c takes units
    // c, c + grid, ... of strip_units.
    int64_t strip_units;
    int strip_pk;
    unsigned long long* timeouts;  // device counter of timed-out waits (async_copy.cuh)
};

struct RedPlan {
    RedPath path = RedPath::Empty;
    RedSpace space;
    RedArgs args;
    int block = 256;
    unsigned grid = 1;
    bool warp_rows = false;  // Inner: one warp per row instead of one CTA per row
    int row_group = 1;       // Inner warp rows: warps sharing one row (1, 2 or 4)
    int col_tile = 0;        // Outer: columns per CTA
    bool bulk = false;       // Outer: bulk-copy column kernel (red_cols_bulk) instead of red_outer
    bool narrow = false;     // Outer: contiguous narrow rows (red_cols_narrow) instead of red_outer
    bool bulk_fixup = false; // bulk: some column tile is shared by several CTAs (second pass)
    bool strip = false;      // Outer: column strips read by tensor copies (red_cols_strip)
    bool runs = false;       // General, CTA per output: the innermost reduced dim is contiguous and
                             // pack-aligned, so red_runs_cta streams 16-byte packs along its runs
    int64_t bulk_tiles = 0;  // bulk: column tiles
    CUtensorMap strip_map;   // strip: the input as a [batch, K, N] tensor of 16-byte-aligned rows
};

// Builds the kept/reduced split of `in` for the given mask and output view(s) (out2 may be null),
// collapses each half, and classifies it. Output strides follow ctorch's rule: with keepdim
// (out rank == in rank) every input dim has an output slot, otherwise only kept dims do
// (src/ops/reduction_iter.cpp:20-69).
int plan_reduction(const ctb_view* in, const ctb_view* out, const ctb_view* out2, uint32_t mask,
                   RedPlan& plan);

// Resident 256-thread CTAs per SM of each reduction kernel (register-limited, so it differs per
// reducer); grids are sized to whole waves of these.
struct RedOcc {
    int inner_cta = 4, inner_warp = 4, outer = 4, general_cta = 4;
    int cols_bulk = 0;  // resident bulk column CTAs per SM; 0 when that kernel cannot take the plan
    int cols_narrow = 0;  // resident narrow-column CTAs per SM; 0 when that kernel cannot take it
    int runs = 0;         // resident red_runs_cta CTAs per SM; 0 when that kernel cannot take the plan
    int cols_strip = 0;   // resident strip column CTAs per SM; 0 when that kernel cannot take it
    int strip_pk_max = 0; // strip: the widest strip in packs (a tensor copy's row is at most 256 elements)
};

// Narrow column kernel: 256 threads, each owning one 16-byte column group of a contiguous
// [K, N] block with N of at most 256 packs.
constexpr int kNarrowBlock = 256;

// Bulk column kernel geometry: each CTA has 8 consumer warps and 1 producer warp. A column tile
// is 4 KiB of a row (256 threads x one 16-byte pack of columns each), a stage holds 8 rows of it,
// and 6 stages (192 KiB) make one CTA per SM. Measured on B200 against 2 KiB tiles with 4
// consumer warps at two CTAs per SM (the same shared memory and consumer threads per SM):
// argmax over dim 0 of [8192, 8192] float32, first pass 47.1 -> 45.7 us.
constexpr int kColsConsumers = 256;
constexpr int kColsRowBytes = 4096;
constexpr int kColsRows = 8;
constexpr int kColsThreads = kColsConsumers + 32;

// Strip column kernel geometry (the same 8 consumer warps and 1 producer warp). A CTA owns a strip
// of whole columns over all K rows, so no second pass combines partial states. Its consumer
// threads form Q = 256 / PK row groups of PK threads (one 16-byte pack of the strip each); a
// stage is one tensor copy of Q * kStripRows rows of the strip (at most 32 KiB), and 4 stages
// are in flight. A tensor copy moves its box row by row, so strips narrower than
// kStripMinPacks (192 bytes) leave the copy engine, not the HBM, as the limit (argmax over dim 0
// of float32 on B200, 268 MB: 71.7 us at 64-byte strips, 44.3-44.9 us at 224-byte strips against
// 49.2 us for the bulk kernel's two passes).
constexpr int kStripStages = 4;
constexpr int kStripRows = 8;
constexpr int kStripStageBytes = kColsConsumers * kStripRows * 16;
constexpr int64_t kStripMinPacks = 12;
constexpr int64_t kStripMinK = 1024;

// Strips per batch row for `batch` rows of `np` packs over `slots` CTAs: the count whose widest
// strip times the rounds of units is least (ties to fewer strips), with strips kStripMinPacks to
// pk_max packs wide. False when none is within 95% of an even spread of the packs over the slots.
bool strip_geometry(int64_t batch, int64_t np, int64_t pk_max, int64_t slots, int64_t& strips, int64_t& pk);

// Chooses split counts / grid for a planned reduction. `state_bytes` is the size of one partial
// state, `outer_vec` the column-strip pack width the Outer kernel will use; returns the scratch
// bytes the plan needs.
size_t finish_reduction_plan(RedPlan& plan, int elem_bytes, int state_bytes, int outer_vec,
                             const RedOcc& occ);

const char* red_path_name(RedPath p);

// The first kernel the calling thread's last reduction launched (a static name), for tests that
// check which kernel a shape takes.
void note_reduction_kernel(const char* name);
const char* last_reduction_kernel();

}  // namespace ctb
