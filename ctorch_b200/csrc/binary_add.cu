// binary_add.cu — instantiates the CTB_ADD dtype dispatch (see binary_impl.cuh).
#include "binary_impl.cuh"

namespace ctb {
template int binary_dispatch<CTB_ADD>(const ctb_view*, const ctb_view*, const ctb_view*, cudaStream_t);
}  // namespace ctb
