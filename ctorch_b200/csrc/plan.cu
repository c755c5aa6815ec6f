// plan.cu — host-side planning for the elementwise and reduction kernels (see plan.cuh).
#include "plan.cuh"

#include <algorithm>
#include <string>

namespace ctb {

const char* ew_path_name(EwPath p) {
    switch (p) {
    case EwPath::Empty: return "empty";
    case EwPath::Flat: return "flat";
    case EwPath::RowsLong: return "rows_long";
    case EwPath::RowsShort: return "rows_short";
    case EwPath::RowsMid: return "rows_mid";
    case EwPath::Tiled: return "tiled";
    case EwPath::General: return "general";
    }
    return "?";
}

const char* red_path_name(RedPath p) {
    switch (p) {
    case RedPath::Empty: return "empty";
    case RedPath::Inner: return "inner";
    case RedPath::Outer: return "outer";
    case RedPath::General: return "general";
    }
    return "?";
}

bool broadcast_strides(const ctb_view& v, int rank, const int64_t* shape, int64_t* strides) {
    if (v.ndim > rank || v.ndim < 0) return false;
    for (int i = 0; i < rank; ++i) {
        const int j = i - (rank - v.ndim);
        if (j < 0) {
            strides[i] = 0;
        } else if (v.shape[j] == shape[i]) {
            strides[i] = v.shape[j] == 1 ? 0 : v.strides[j];
        } else if (v.shape[j] == 1) {
            strides[i] = 0;
        } else {
            return false;
        }
    }
    return true;
}

void collapse(EwSpace& s) {
    // 1) drop size-1 dims
    EwSpace t;
    t.nops = s.nops;
    for (int d = 0; d < s.rank; ++d) {
        if (s.shape[d] == 1) continue;
        t.shape[t.rank] = s.shape[d];
        for (int o = 0; o < s.nops; ++o) t.stride[o][t.rank] = s.stride[o][d];
        ++t.rank;
    }
    if (t.rank == 0) {
        t.rank = 1;
        t.shape[0] = 1;
        for (int o = 0; o < s.nops; ++o) t.stride[o][0] = 0;
        s = t;
        return;
    }
    // 2) merge d into d+1 (walking outward) when every operand's strides chain
    EwSpace m;
    m.nops = t.nops;
    m.rank = 1;
    // build innermost-first, then reverse
    int64_t shp[kMaxDims];
    int64_t st[kMaxOps][kMaxDims];
    int r = 0;
    shp[0] = t.shape[t.rank - 1];
    for (int o = 0; o < t.nops; ++o) st[o][0] = t.stride[o][t.rank - 1];
    r = 1;
    for (int d = t.rank - 2; d >= 0; --d) {
        bool chain = true;
        for (int o = 0; o < t.nops; ++o)
            if (t.stride[o][d] != st[o][r - 1] * shp[r - 1]) chain = false;
        if (chain) {
            shp[r - 1] *= t.shape[d];
        } else {
            shp[r] = t.shape[d];
            for (int o = 0; o < t.nops; ++o) st[o][r] = t.stride[o][d];
            ++r;
        }
    }
    m.rank = r;
    for (int i = 0; i < r; ++i) {
        m.shape[i] = shp[r - 1 - i];
        for (int o = 0; o < t.nops; ++o) m.stride[o][i] = st[o][r - 1 - i];
    }
    s = m;
}

// Reorders dims so that out's strides are non-increasing (stable). Elementwise results do not
// depend on iteration order, and this puts out's unit-stride dim innermost when out is a
// permuted view (in-place ops on non-contiguous tensors).
static void order_by_out(EwSpace& s) {
    int perm[kMaxDims];
    for (int d = 0; d < s.rank; ++d) perm[d] = d;
    std::stable_sort(perm, perm + s.rank, [&](int x, int y) {
        const int64_t ax = s.stride[0][x] < 0 ? -s.stride[0][x] : s.stride[0][x];
        const int64_t ay = s.stride[0][y] < 0 ? -s.stride[0][y] : s.stride[0][y];
        return ax > ay;
    });
    EwSpace t = s;
    for (int d = 0; d < s.rank; ++d) {
        t.shape[d] = s.shape[perm[d]];
        for (int o = 0; o < s.nops; ++o) t.stride[o][d] = s.stride[o][perm[d]];
    }
    s = t;
}

int plan_elementwise(const ctb_view* out, const ctb_view* const* ins, int nin, const int* sizes,
                     int vec, EwPlan& plan) {
    if (out->ndim < 0 || out->ndim > kMaxDims)
        return fail(CTB_ERR_SHAPE, "rank exceeds " + std::to_string(kMaxDims));
    for (int i = 0; i < nin; ++i)
        if (ins[i]->ndim < 0 || ins[i]->ndim > kMaxDims)
            return fail(CTB_ERR_SHAPE, "rank exceeds " + std::to_string(kMaxDims));
    EwSpace& s = plan.space;
    s = EwSpace{};
    s.nops = 1 + nin;
    s.rank = out->ndim;
    for (int d = 0; d < s.rank; ++d) {
        if (out->shape[d] < 0) return fail(CTB_ERR_SHAPE, "negative extent");
        s.shape[d] = out->shape[d];
        s.stride[0][d] = out->strides[d];
    }
    for (int i = 0; i < nin; ++i) {
        if (!broadcast_strides(*ins[i], s.rank, s.shape, s.stride[1 + i]))
            return fail(CTB_ERR_SHAPE, "operand shape does not broadcast to the output shape");
    }
    plan.vec = vec;
    if (s.numel() == 0) {
        plan.path = EwPath::Empty;
        return CTB_OK;
    }
    order_by_out(s);
    collapse(s);

    EwArgs& a = plan.args;
    a = EwArgs{};
    a.out = out->data;
    for (int i = 0; i < nin; ++i) a.in[i] = ins[i]->data;
    a.rank = s.rank;
    a.n = s.numel();
    a.L = s.shape[s.rank - 1];
    a.rows = a.n / a.L;
    for (int d = 0; d < s.rank; ++d) {
        a.shape[d] = s.shape[d];
        a.div[d] = FastDiv(static_cast<uint64_t>(s.shape[d]));
        for (int o = 0; o < s.nops; ++o) a.stride[o][d] = s.stride[o][d];
    }

    const int r = s.rank;
    const void* base[kMaxOps] = {out->data, nin > 0 ? ins[0]->data : nullptr,
                                 nin > 1 ? ins[1]->data : nullptr, nin > 2 ? ins[2]->data : nullptr};
    bool inner_ok = s.stride[0][r - 1] == 1;
    for (int o = 1; o < s.nops; ++o) inner_ok = inner_ok && (s.stride[o][r - 1] == 0 || s.stride[o][r - 1] == 1);

    // Vector alignment: every operand read with unit inner stride must start each vector on a
    // 16-byte boundary: base aligned and every outer stride a whole number of 16-byte chunks.
    bool aligned = true;
    for (int o = 0; o < s.nops && aligned; ++o) {
        if (s.stride[o][r - 1] != 1) continue;
        if (!aligned16(base[o])) aligned = false;
        for (int d = 0; d < r - 1; ++d)
            if ((s.stride[o][d] * sizes[o]) % 16 != 0) aligned = false;
    }

    if (inner_ok && aligned && r == 1) {
        plan.path = EwPath::Flat;
        return CTB_OK;
    }
    if (inner_ok && aligned && a.L % vec == 0) {
        a.vpr = a.L / vec;
        if (a.vpr >= kRowsLongPacks) {
            a.aux = FastDiv(static_cast<uint64_t>((a.vpr + kRowsLongPacks - 1) / kRowsLongPacks));
            plan.path = EwPath::RowsLong;
        } else if (a.vpr >= kRowsMidPacks) {
            a.aux = FastDiv(static_cast<uint64_t>((a.vpr + kRowsMidPacks - 1) / kRowsMidPacks));
            plan.path = EwPath::RowsMid;
        } else {
            a.aux = FastDiv(static_cast<uint64_t>(a.vpr));
            plan.path = EwPath::RowsShort;
        }
        return CTB_OK;
    }
    // Tiled transpose: exactly one input walks the inner dim with a stride other than 0/1 but has
    // unit stride on some outer dim p; everything else is unit/zero stride on the inner dim.
    if (r >= 2 && s.stride[0][r - 1] == 1 && a.L >= 8) {
        int xop = -1, pdim = -1, others_ok = 1;
        for (int o = 1; o < s.nops; ++o) {
            const int64_t st = s.stride[o][r - 1];
            if (st == 0 || st == 1) continue;
            if (xop != -1) { others_ok = 0; break; }
            for (int d = r - 2; d >= 0; --d)
                if (s.stride[o][d] == 1 && s.shape[d] >= 8) { pdim = d; break; }
            xop = o;
        }
        if (others_ok && xop != -1 && pdim != -1) {
            a.xop = xop;
            a.pdim = pdim;
            // 4-element packs: every operand's base aligned to its pack (16 B for 4-byte types,
            // 32 B for 8-byte types -> 16 B suffices for whole-chunk access), the row-major input
            // unit-stride on the inner dim, and every other stride a multiple of 4 elements.
            const int yop = xop == 1 ? (s.nops > 2 ? 2 : -1) : 1;
            bool v4 = yop > 0 && s.stride[yop][r - 1] == 1;
            for (int o = 0; o < s.nops && v4; ++o) {
                if (!aligned16(base[o])) v4 = false;
                for (int d = 0; d < r; ++d) {
                    const int64_t st = s.stride[o][d];
                    const bool unit = (o == xop && d == pdim) || (o != xop && d == r - 1);
                    if (!unit && st % 4 != 0) v4 = false;
                }
            }
            a.tiled_vec = v4 ? 1 : 0;
            constexpr int kTile = 64;
            a.aux = FastDiv(static_cast<uint64_t>((a.L + kTile - 1) / kTile));
            a.aux2 = FastDiv(static_cast<uint64_t>((s.shape[pdim] + kTile - 1) / kTile));
            // batch dims: all dims except pdim and the inner one
            plan.path = EwPath::Tiled;
            return CTB_OK;
        }
    }
    plan.path = EwPath::General;
    return CTB_OK;
}

// ------------------------------------------------------------------------------------------------

int plan_reduction(const ctb_view* in, const ctb_view* out, const ctb_view* out2, uint32_t mask,
                   RedPlan& plan) {
    const int rank = in->ndim;
    if (rank < 0 || rank > kMaxDims) return fail(CTB_ERR_SHAPE, "rank exceeds 16");
    if (rank < 32 && (mask >> rank) != 0u) return fail(CTB_ERR_SHAPE, "reduction axis out of range");
    int n_kept = 0;
    for (int d = 0; d < rank; ++d)
        if (!((mask >> d) & 1u)) ++n_kept;
    const bool keepdim = out->ndim == rank;
    if (!keepdim && out->ndim != n_kept)
        return fail(CTB_ERR_SHAPE, "output rank matches neither keepdim nor dropped layout");
    if (out2 && out2->ndim != out->ndim) return fail(CTB_ERR_SHAPE, "values/indices rank differ");

    RedSpace raw;
    int od = 0;
    for (int d = 0; d < rank; ++d) {
        const bool red = (mask >> d) & 1u;
        if (in->shape[d] < 0) return fail(CTB_ERR_SHAPE, "negative extent");
        if (red) {
            if (keepdim && out->shape[od] != 1) return fail(CTB_ERR_SHAPE, "keepdim output must be 1 at reduced dims");
            if (keepdim && out2 && out2->shape[od] != 1) return fail(CTB_ERR_SHAPE, "keepdim output must be 1 at reduced dims");
            raw.shape_r[raw.rank_r] = in->shape[d];
            raw.stride_r[raw.rank_r] = in->strides[d];
            raw.red *= in->shape[d];
            ++raw.rank_r;
        } else {
            if (out->shape[od] != in->shape[d]) return fail(CTB_ERR_SHAPE, "output shape mismatch");
            if (out2 && out2->shape[od] != in->shape[d]) return fail(CTB_ERR_SHAPE, "index output shape mismatch");
            raw.shape_k[raw.rank_k] = in->shape[d];
            raw.stride_k[raw.rank_k] = in->strides[d];
            raw.stride_o[raw.rank_k] = out->strides[od];
            raw.stride_o2[raw.rank_k] = out2 ? out2->strides[od] : 0;
            raw.kept *= in->shape[d];
            ++raw.rank_k;
        }
        if (keepdim || !red) ++od;
    }

    // Collapse the kept half (three stride sets) and the reduced half (one), innermost first.
    RedSpace& s = plan.space;
    s = RedSpace{};
    s.kept = raw.kept;
    s.red = raw.red;
    {
        int64_t shp[kMaxDims], sk[kMaxDims], so[kMaxDims], so2[kMaxDims];
        int r = 0;
        for (int d = raw.rank_k - 1; d >= 0; --d) {
            if (raw.shape_k[d] == 1) continue;
            if (r > 0 && raw.stride_k[d] == sk[r - 1] * shp[r - 1] &&
                raw.stride_o[d] == so[r - 1] * shp[r - 1] &&
                raw.stride_o2[d] == so2[r - 1] * shp[r - 1]) {
                shp[r - 1] *= raw.shape_k[d];
            } else {
                shp[r] = raw.shape_k[d];
                sk[r] = raw.stride_k[d];
                so[r] = raw.stride_o[d];
                so2[r] = raw.stride_o2[d];
                ++r;
            }
        }
        s.rank_k = r;
        for (int i = 0; i < r; ++i) {
            s.shape_k[i] = shp[r - 1 - i];
            s.stride_k[i] = sk[r - 1 - i];
            s.stride_o[i] = so[r - 1 - i];
            s.stride_o2[i] = so2[r - 1 - i];
        }
    }
    {
        int64_t shp[kMaxDims], sr[kMaxDims];
        int r = 0;
        for (int d = raw.rank_r - 1; d >= 0; --d) {
            if (raw.shape_r[d] == 1) continue;
            if (r > 0 && raw.stride_r[d] == sr[r - 1] * shp[r - 1]) {
                shp[r - 1] *= raw.shape_r[d];
            } else {
                shp[r] = raw.shape_r[d];
                sr[r] = raw.stride_r[d];
                ++r;
            }
        }
        s.rank_r = r;
        for (int i = 0; i < r; ++i) {
            s.shape_r[i] = shp[r - 1 - i];
            s.stride_r[i] = sr[r - 1 - i];
        }
    }

    RedArgs& a = plan.args;
    a = RedArgs{};
    a.in = in->data;
    a.out = out->data;
    a.out2 = out2 ? out2->data : nullptr;
    a.rank_k = s.rank_k;
    a.rank_r = s.rank_r;
    a.kept = s.kept;
    a.red = s.red;
    for (int i = 0; i < s.rank_k; ++i) {
        a.shape_k[i] = s.shape_k[i];
        a.stride_k[i] = s.stride_k[i];
        a.stride_o[i] = s.stride_o[i];
        a.stride_o2[i] = s.stride_o2[i];
        a.div_k[i] = FastDiv(static_cast<uint64_t>(s.shape_k[i]));
    }
    for (int i = 0; i < s.rank_r; ++i) {
        a.shape_r[i] = s.shape_r[i];
        a.stride_r[i] = s.stride_r[i];
        a.div_r[i] = FastDiv(static_cast<uint64_t>(s.shape_r[i]));
    }

    if (s.kept == 0) {
        plan.path = RedPath::Empty;
        return CTB_OK;
    }
    if (s.red == 0) {
        plan.path = RedPath::General;  // writes the identity everywhere
        return CTB_OK;
    }
    if (s.rank_r == 1 && s.stride_r[0] == 1) {
        plan.path = RedPath::Inner;
        a.K = s.shape_r[0];
        return CTB_OK;
    }
    if (s.rank_r == 1 && s.rank_k >= 1 && s.stride_k[s.rank_k - 1] == 1 &&
        s.stride_o[s.rank_k - 1] == 1 && (!out2 || s.stride_o2[s.rank_k - 1] == 1) &&
        s.shape_k[s.rank_k - 1] >= 16) {
        plan.path = RedPath::Outer;
        a.N = s.shape_k[s.rank_k - 1];
        a.K = s.shape_r[0];
        a.strideK = s.stride_r[0];
        return CTB_OK;
    }
    plan.path = RedPath::General;
    return CTB_OK;
}

// Split count in [1, max_split] whose CTAs (tiles * split) fill one or two whole waves of `slots`
// best; a larger split must fill at least 2% more to be chosen (it costs partial-state traffic).
static int64_t best_split(int64_t tiles, int64_t slots, int64_t max_split) {
    int64_t best = 1;
    double best_fill = -1.0;
    const int64_t hi = std::max<int64_t>(1, std::min<int64_t>(max_split, 2 * slots / std::max<int64_t>(1, tiles)));
    for (int64_t s = 1; s <= hi; ++s) {
        const int64_t ctas = tiles * s;
        const int64_t waves = (ctas + slots - 1) / slots;
        const double fill = static_cast<double>(ctas) / static_cast<double>(waves * slots);
        if (fill > best_fill + 0.02) {
            best_fill = fill;
            best = s;
        }
    }
    return best;
}

namespace {
thread_local const char* g_last_reduction_kernel = "";
}

void note_reduction_kernel(const char* name) { g_last_reduction_kernel = name; }
const char* last_reduction_kernel() { return g_last_reduction_kernel; }

bool strip_geometry(int64_t batch, int64_t np, int64_t pk_max, int64_t slots, int64_t& strips, int64_t& pk) {
    if (batch < 1 || np < kStripMinPacks || pk_max < kStripMinPacks || slots < 1) return false;
    const int64_t lo = (np + pk_max - 1) / pk_max;  // fewest strips a row can have
    const int64_t hi = std::min(np / kStripMinPacks, lo + 4 * slots);
    int64_t best = 0, best_cost = 0;
    for (int64_t s = lo; s <= hi; ++s) {
        // time of the busiest CTA, in pack-rows: its rounds of units times the widest strip
        const int64_t cost = ((batch * s + slots - 1) / slots) * ((np + s - 1) / s);
        if (best == 0 || cost < best_cost) {
            best = s;
            best_cost = cost;
        }
    }
    if (best == 0) return false;
    // an even spread of every pack-row over the slots
    const double ideal = static_cast<double>(batch) * static_cast<double>(np) / static_cast<double>(slots);
    if (ideal < 0.95 * static_cast<double>(best_cost)) return false;
    strips = best;
    pk = (np + best - 1) / best;
    return true;
}

size_t finish_reduction_plan(RedPlan& plan, int elem_bytes, int state_bytes, int outer_vec,
                             const RedOcc& occ) {
    RedArgs& a = plan.args;
    const int64_t sms = sm_count();
    plan.block = 256;
    plan.bulk = false;
    plan.narrow = false;
    plan.row_group = 1;
    plan.bulk_fixup = false;
    plan.runs = false;
    plan.strip = false;
    a.split = 1;
    a.chunk = a.red;
    a.sk_q = a.sk_r = 0;
    size_t scratch = 0;
    switch (plan.path) {
    case RedPath::Empty:
        plan.grid = 0;
        break;
    case RedPath::Inner: {
        const int64_t K = a.K;
        if (K <= 65536 && a.kept >= sms * 16) {
            // one warp per row (or a group of 2 or 4 warps per long row when there are fewer than
            // ~6 rows per resident warp), persistent grid of one wave
            plan.warp_rows = true;
            const int64_t slots = sms * occ.inner_warp;
            const int64_t warps = slots * 8;
            plan.row_group = 1;
            if (K * elem_bytes > 8192) {
                while (plan.row_group < 4 && a.kept * plan.row_group < 6 * warps) plan.row_group *= 2;
            }
            // as many rounds of rows as a full wave needs, and just enough CTAs for them, so that
            // the last round is as full as the others
            const int64_t rows_per_cta = 8 / plan.row_group;
            const int64_t wave = slots * rows_per_cta;
            const int64_t rounds = (a.kept + wave - 1) / wave;
            const int64_t rows_per_round = (a.kept + rounds - 1) / rounds;
            const int64_t ctas = (rows_per_round + rows_per_cta - 1) / rows_per_cta;
            plan.grid = static_cast<unsigned>(ctas < slots ? ctas : slots);
            break;
        }
        plan.warp_rows = false;
        const int64_t slots = sms * occ.inner_cta;
        int64_t split = 1;
        if (a.kept < slots) {
            split = slots / a.kept;
            split = std::min<int64_t>(split, std::max<int64_t>(1, K / 4096));
            split = std::max<int64_t>(split, 1);
        }
        // chunks are whole 64-byte multiples so every split starts 16-byte aligned when the row does
        int64_t chunk = (K + split - 1) / split;
        const int64_t q = 64 / elem_bytes > 0 ? 64 / elem_bytes : 1;
        chunk = (chunk + q - 1) / q * q;
        split = (K + chunk - 1) / chunk;
        a.split = static_cast<int>(split);
        a.chunk = chunk;
        a.aux = FastDiv(static_cast<uint64_t>(split));
        const int64_t work = a.kept * split;
        plan.grid = static_cast<unsigned>(work < slots ? work : slots);
        if (split > 1) scratch = static_cast<size_t>(a.kept * split) * state_bytes;
        break;
    }
    case RedPath::Outer: {
        if (occ.cols_narrow > 0) {
            // one CTA streams a contiguous block of whole rows; the rows are split over CTAs to fill
            // the GPU, and the splits of each output are combined in order by red_finalize
            plan.narrow = true;
            plan.block = kNarrowBlock;
            const int64_t vec = 16 / elem_bytes;
            const int64_t np = a.N / vec;
            const int64_t lanes = std::max<int64_t>(1, kNarrowBlock / np);
            const int64_t tiles = a.kept / a.N;
            const int64_t slots = sms * occ.cols_narrow;
            int64_t split = 1;
            const int64_t cap = std::max<int64_t>(1, (int64_t(4) << 20) / std::max<int64_t>(1, a.kept * state_bytes));
            const int64_t max_split = std::max<int64_t>(1, std::min(a.K / (4 * lanes), cap));
            if (tiles < 2 * slots) split = best_split(tiles, slots, max_split);
            constexpr int64_t kMaxChunk = (int64_t(1) << 31) - 2;
            split = std::max<int64_t>(split, (a.K + kMaxChunk - 1) / kMaxChunk);
            int64_t chunk = (a.K + split - 1) / split;
            split = (a.K + chunk - 1) / chunk;
            a.split = static_cast<int>(split);
            a.chunk = chunk;
            a.aux2 = FastDiv(static_cast<uint64_t>(split));
            const int64_t work = tiles * split;
            plan.grid = static_cast<unsigned>(work < slots ? work : slots);
            if (split > 1) scratch = static_cast<size_t>(a.kept * split) * state_bytes;
            break;
        }
        if (occ.cols_strip > 0) {
            // whole columns per CTA: a batch row's packs cut into strips, one unit per (batch row,
            // strip), units spread evenly over one CTA per SM
            const int64_t vec = 16 / elem_bytes;
            const int64_t batch = a.kept / a.N;
            int64_t strips = 0, pk = 0;
            if (strip_geometry(batch, a.N / vec, occ.strip_pk_max, sms * occ.cols_strip, strips, pk)) {
                plan.strip = true;
                plan.block = kColsThreads;
                a.aux = FastDiv(static_cast<uint64_t>(strips));
                a.strip_units = batch * strips;
                a.strip_pk = static_cast<int>(pk);
                const int64_t slots = sms * occ.cols_strip;
                plan.grid = static_cast<unsigned>(a.strip_units < slots ? a.strip_units : slots);
                break;
            }
        }
        if (occ.cols_bulk > 0) {
            // Stream-K over (column tile, row): G CTAs take equal shares of the row-steps, so
            // every CTA streams the same number of bytes whatever the tile count; a tile shared
            // by several CTAs is combined in CTA order by red_cols_finalize.
            plan.bulk = true;
            plan.block = kColsThreads;
            const int64_t tw = kColsRowBytes / elem_bytes;  // columns per tile
            const int64_t tiles_n = (a.N + tw - 1) / tw;
            const int64_t tiles = tiles_n * (a.kept / a.N);
            const int64_t steps = tiles * a.K;
            const int64_t slots = sms * occ.cols_bulk;
            // partial states (one row of tw per CTA-and-tile pair, G + tiles - 1 pairs at most)
            // are held to 4 MiB
            const int64_t cap = std::max<int64_t>(1, (int64_t(4) << 20) / (tw * state_bytes) - tiles);
            int64_t G = std::min<int64_t>({slots, cap, std::max<int64_t>(1, steps / (2 * kColsRows))});
            G = std::max<int64_t>(1, std::min<int64_t>(G, steps));
            a.sk_q = steps / G;
            a.sk_r = steps % G;
            a.aux = FastDiv(static_cast<uint64_t>(tiles_n));
            a.aux2 = FastDiv(static_cast<uint64_t>(a.K));
            plan.grid = static_cast<unsigned>(G);
            plan.bulk_tiles = tiles;
            plan.bulk_fixup = false;
            for (int64_t c = 1; c < G && !plan.bulk_fixup; ++c)
                if ((c * a.sk_q + std::min<int64_t>(c, a.sk_r)) % a.K != 0) plan.bulk_fixup = true;
            if (plan.bulk_fixup) scratch = static_cast<size_t>(G + tiles) * tw * state_bytes;
            break;
        }
        plan.col_tile = 32 * outer_vec;
        const int64_t tiles_n = (a.N + plan.col_tile - 1) / plan.col_tile;
        const int64_t batch = a.kept / a.N;
        const int64_t tiles = tiles_n * batch;
        const int64_t slots = sms * occ.outer;
        int64_t split = 1;
        // partials are kept to 2 MiB: at most a few percent of the bytes the reduction reads
        const int64_t cap = std::max<int64_t>(1, (int64_t(2) << 20) / std::max<int64_t>(1, a.kept * state_bytes));
        if (tiles < 2 * slots) split = best_split(tiles, slots, std::max<int64_t>(1, std::min(a.K / 64, cap)));
        // the kernel folds positions as 32-bit offsets within a chunk
        constexpr int64_t kMaxChunk = (int64_t(1) << 31) - 2;
        split = std::max<int64_t>(split, (a.K + kMaxChunk - 1) / kMaxChunk);
        int64_t chunk = (a.K + split - 1) / split;
        split = (a.K + chunk - 1) / chunk;
        a.split = static_cast<int>(split);
        a.chunk = chunk;
        a.aux = FastDiv(static_cast<uint64_t>(tiles_n));
        a.aux2 = FastDiv(static_cast<uint64_t>(split));
        const int64_t work = tiles * split;
        plan.grid = static_cast<unsigned>(work < slots ? work : slots);
        if (split > 1) scratch = static_cast<size_t>(a.kept * split) * state_bytes;
        break;
    }
    case RedPath::General: {
        const int64_t slots = sms * occ.general_cta;
        // few outputs with long reduced ranges: CTAs share an output; otherwise one thread each
        if (a.kept < slots * 32 && a.red >= 1024) {
            // contiguous innermost reduced dim, whole packs per run, runs on 16-byte boundaries:
            // red_runs_cta (chunks counted in packs) instead of the per-element decode
            const int vec = 16 / elem_bytes;
            const int64_t run = a.rank_r > 0 ? a.shape_r[a.rank_r - 1] : 0;
            const int64_t rslots = sms * occ.runs;
            bool runs = occ.runs > 0 && a.rank_r > 0 && a.stride_r[a.rank_r - 1] == 1 &&
                        run % vec == 0 && run >= 4 * vec && reinterpret_cast<uintptr_t>(a.in) % 16 == 0;
            for (int d = 0; runs && d < a.rank_k; ++d) runs = (a.stride_k[d] * elem_bytes) % 16 == 0;
            for (int d = 0; runs && d + 1 < a.rank_r; ++d) runs = (a.stride_r[d] * elem_bytes) % 16 == 0;
            const int64_t units = runs ? a.red / vec : a.red;  // packs or elements
            const int64_t use_slots = runs ? rslots : slots;
            int64_t split = std::max<int64_t>(1, use_slots / a.kept);
            split = std::min<int64_t>(split, std::max<int64_t>(1, a.red / 4096));
            const int64_t chunk = (units + split - 1) / split;
            split = (units + chunk - 1) / chunk;
            a.split = static_cast<int>(split);
            a.chunk = chunk;
            a.aux = FastDiv(static_cast<uint64_t>(split));
            if (runs) a.aux2 = FastDiv(static_cast<uint64_t>(run / vec));
            plan.runs = runs;
            plan.warp_rows = false;
            const int64_t work = a.kept * split;
            plan.grid = static_cast<unsigned>(work < use_slots ? work : use_slots);
            if (split > 1) scratch = static_cast<size_t>(a.kept * split) * state_bytes;
        } else {
            plan.warp_rows = true;  // here: one thread per output
            plan.grid = grid_for((a.kept + 255) / 256, 32);
        }
        break;
    }
    }
    return scratch;
}

}  // namespace ctb
