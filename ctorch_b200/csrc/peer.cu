// peer.cu — host side of the cross-GPU one-pass sum: the per-rank workspace (allocation, CUDA IPC
// export and import). The launch itself is ctb_chain_rows_allsum (capi.cu, fused_rows.cu).
#include <cstddef>
#include <cstring>
#include <string>

#include "common.cuh"
#include "peer.cuh"

namespace ctb {

namespace {
int cuda_fail(const char* what, cudaError_t e) {
    cudaGetLastError();
    return fail(CTB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}
}  // namespace

}  // namespace ctb

using namespace ctb;

extern "C" {

CTB_API size_t ctb_peer_workspace_bytes(void) { return sizeof(PeerWorkspace); }

CTB_API int ctb_peer_alloc(void** d_workspace, void* ipc_handle) {
    if (!d_workspace || !ipc_handle) return fail(CTB_ERR_ARGUMENT, "ctb_peer_alloc: null argument");
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, sizeof(PeerWorkspace));
    if (e != cudaSuccess) return cuda_fail("ctb_peer_alloc: cudaMalloc", e);
    e = cudaMemset(p, 0, sizeof(PeerWorkspace));
    if (e == cudaSuccess) {
        cudaIpcMemHandle_t h;
        e = cudaIpcGetMemHandle(&h, p);
        if (e == cudaSuccess) {
            std::memcpy(ipc_handle, &h, sizeof(h));
            *d_workspace = p;
            return CTB_OK;
        }
    }
    cudaFree(p);
    return cuda_fail("ctb_peer_alloc", e);
}

CTB_API int ctb_peer_open(const void* ipc_handle, void** d_peer_workspace) {
    if (!ipc_handle || !d_peer_workspace) return fail(CTB_ERR_ARGUMENT, "ctb_peer_open: null argument");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, ipc_handle, sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail("ctb_peer_open: cudaIpcOpenMemHandle", e);
    *d_peer_workspace = p;
    return CTB_OK;
}

CTB_API int ctb_peer_close(void* d_peer_workspace) {
    const cudaError_t e = cudaIpcCloseMemHandle(d_peer_workspace);
    return e == cudaSuccess ? CTB_OK : cuda_fail("ctb_peer_close", e);
}

CTB_API int ctb_peer_status(const void* d_my_workspace, uint64_t* done_epoch, uint64_t* failed_epoch) {
    if (!d_my_workspace || !done_epoch || !failed_epoch) return fail(CTB_ERR_ARGUMENT, "ctb_peer_status: null argument");
    uint64_t st[2];
    const cudaError_t e = cudaMemcpy(st, static_cast<const char*>(d_my_workspace) + offsetof(PeerWorkspace, done_epoch),
                                     sizeof(st), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail("ctb_peer_status", e);
    static_assert(offsetof(PeerWorkspace, failed_epoch) == offsetof(PeerWorkspace, done_epoch) + 8, "layout");
    *done_epoch = st[0];
    *failed_epoch = st[1];
    return CTB_OK;
}

CTB_API int ctb_peer_trace(const void* d_my_workspace, uint64_t* out) {
    if (!d_my_workspace || !out) return fail(CTB_ERR_ARGUMENT, "ctb_peer_trace: null argument");
    const cudaError_t e = cudaMemcpy(out, static_cast<const char*>(d_my_workspace) + offsetof(PeerWorkspace, trace),
                                     sizeof(PeerWorkspace::trace), cudaMemcpyDeviceToHost);
    return e == cudaSuccess ? CTB_OK : cuda_fail("ctb_peer_trace", e);
}

CTB_API int ctb_peer_free(void* d_workspace) {
    const cudaError_t e = cudaFree(d_workspace);
    return e == cudaSuccess ? CTB_OK : cuda_fail("ctb_peer_free", e);
}

}  // extern "C"
