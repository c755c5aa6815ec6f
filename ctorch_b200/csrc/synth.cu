// synth.cu — counter-based synthetic inputs: element i of (seed, stream) gets
// h = splitmix64(key + i), key = splitmix64(splitmix64(seed) ^ stream). Uniform floats use the top
// 24 bits, lo + (hi - lo) * u in double rounded once to the dtype; integer uniforms use
// lo + h mod (hi - lo + 1); normals use Box-Muller on two 53-bit uniforms. The same (seed,
// stream, global index) always gives the same value, however a tensor is sharded.
#include "common.cuh"

namespace ctb {

__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    uint64_t z = x + 0x9e3779b97f4a7c15ULL;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}

template <class T>
__global__ void fill_kernel(T* out, int64_t n, int dist, uint64_t key, int64_t first, double lo, double hi) {
    dependent_wait();  // the previous kernel in the stream has completed and its writes are visible
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nthr = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = tid; i < n; i += nthr) {
        const uint64_t h = splitmix64(key + static_cast<uint64_t>(first + i));
        if constexpr (is_float_v<T>) {
            double v;
            if (dist == 0) {
                const double u = static_cast<double>(h >> 40) * 0x1.0p-24;
                v = __dadd_rn(lo, __dmul_rn(hi - lo, u));
            } else {
                const double u1 = static_cast<double>((h >> 11) + 1) * 0x1.0p-53;
                const double u2 = static_cast<double>(splitmix64(h) >> 11) * 0x1.0p-53;
                const double z = sqrt(-2.0 * log(u1)) * cospi(2.0 * u2);
                v = __dadd_rn(lo, __dmul_rn(hi, z));
            }
            out[i] = static_cast<T>(v);
        } else {
            const int64_t a = static_cast<int64_t>(lo), b = static_cast<int64_t>(hi);
            const uint64_t range = static_cast<uint64_t>(b - a) + 1;
            const uint64_t r = range == 0 ? h : h % range;
            out[i] = static_cast<T>(static_cast<int64_t>(static_cast<uint64_t>(a) + r));
        }
    }
    allow_dependents();  // the next kernel in the stream may launch while this one winds down
}

int fill_random(const ctb_view* out, int dist, uint64_t seed, uint64_t stream_id, int64_t first,
                double lo, double hi, cudaStream_t st) {
    int64_t n = 1;
    int64_t expect = 1;
    for (int d = out->ndim - 1; d >= 0; --d) {
        if (out->shape[d] != 1 && out->strides[d] != expect)
            return fail(CTB_ERR_SHAPE, "ctb_fill_random needs a contiguous view");
        expect *= out->shape[d];
        n *= out->shape[d];
    }
    if (n == 0) return CTB_OK;
    const uint64_t key = splitmix64(splitmix64(seed) ^ stream_id);
    const unsigned grid = grid_for((n + 255) / 256, 16);
    switch (out->dtype) {
    case CTB_FLOAT32: launch_dependent(fill_kernel<float>, grid, 256, 0, st, static_cast<float*>(out->data), n, dist, key, first, lo, hi); break;
    case CTB_FLOAT64: launch_dependent(fill_kernel<double>, grid, 256, 0, st, static_cast<double*>(out->data), n, dist, key, first, lo, hi); break;
    case CTB_INT32:
        if (dist != 0) return fail(CTB_ERR_DTYPE, "normal fill needs a float dtype");
        launch_dependent(fill_kernel<int32_t>, grid, 256, 0, st, static_cast<int32_t*>(out->data), n, dist, key, first, lo, hi); break;
    case CTB_INT64:
        if (dist != 0) return fail(CTB_ERR_DTYPE, "normal fill needs a float dtype");
        launch_dependent(fill_kernel<int64_t>, grid, 256, 0, st, static_cast<int64_t*>(out->data), n, dist, key, first, lo, hi); break;
    default: return fail(CTB_ERR_DTYPE, "unsupported fill dtype");
    }
    count_launch();
    return check_launch("fill_random");
}

}  // namespace ctb
