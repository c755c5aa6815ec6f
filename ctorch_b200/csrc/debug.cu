// debug.cu — host-only planning introspection (include/ctb/ctb_debug.h). Runs the same planner
// the launches use and reports its decision; makes no CUDA call that needs a device.
#include <cstring>
#include <string>

#include "ctb/ctb_debug.h"
#include "common.cuh"
#include "plan.cuh"

using namespace ctb;

static void put(char* buf, int len, const char* s) {
    if (!buf || len <= 0) return;
    std::strncpy(buf, s, static_cast<size_t>(len - 1));
    buf[len - 1] = '\0';
}

extern "C" {

int ctb_debug_plan_elementwise(const ctb_view* out, const ctb_view* const* ins, int nin, int vec,
                               char* path, int path_len, int* rank, int64_t* shape) {
    if (!out || !ins || nin < 1 || nin > 3) return CTB_ERR_ARGUMENT;
    int sizes[4] = {static_cast<int>(dtype_size(out->dtype)), 0, 0, 0};
    for (int i = 0; i < nin; ++i) sizes[1 + i] = static_cast<int>(dtype_size(ins[i]->dtype));
    EwPlan plan;
    const int rc = plan_elementwise(out, ins, nin, sizes, vec, plan);
    if (rc) return rc;
    put(path, path_len, ew_path_name(plan.path));
    if (rank) *rank = plan.space.rank;
    if (shape)
        for (int d = 0; d < plan.space.rank; ++d) shape[d] = plan.space.shape[d];
    return CTB_OK;
}

int ctb_debug_plan_reduction(const ctb_view* in, const ctb_view* out, uint32_t mask, char* path,
                             int path_len, int* rank_kept, int* rank_red) {
    if (!in || !out) return CTB_ERR_ARGUMENT;
    RedPlan plan;
    const int rc = plan_reduction(in, out, nullptr, mask, plan);
    if (rc) return rc;
    put(path, path_len, red_path_name(plan.path));
    if (rank_kept) *rank_kept = plan.space.rank_k;
    if (rank_red) *rank_red = plan.space.rank_r;
    return CTB_OK;
}

int ctb_debug_strip_geometry(int64_t batch, int64_t np, int64_t pk_max, int64_t slots, int64_t* strips,
                             int64_t* pk) {
    int64_t s = 0, w = 0;
    const bool ok = strip_geometry(batch, np, pk_max, slots, s, w);
    if (strips) *strips = ok ? s : 0;
    if (pk) *pk = ok ? w : 0;
    return ok ? 1 : 0;
}

int ctb_debug_last_reduction_kernel(char* buf, int len) {
    if (!buf || len <= 0) return CTB_ERR_ARGUMENT;
    put(buf, len, last_reduction_kernel());
    return CTB_OK;
}

uint64_t ctb_debug_fastdiv(uint64_t n, uint64_t d) { return FastDiv(d).div(n); }

}  // extern "C"
