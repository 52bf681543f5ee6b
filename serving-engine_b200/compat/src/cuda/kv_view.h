// compat/src/cuda/kv_view.h -- engine::cuda::KVView over b2engine.
//
// Same fields, order and aggregate initialisation as the reference's view
// (src/cuda/kv_view.h:17-31) so its callers build views unchanged; it maps
// field for field onto b2_kv_view at the C-ABI.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

namespace engine {
namespace cuda {

struct KVView {
    const half* __restrict__ data;
    int64_t stride_b;
    int64_t stride_h;
    int64_t stride_s;
    int64_t stride_d;

#ifdef __CUDACC__
    __device__ __forceinline__ const half* get_ptr(int b, int h, int s) const {
        return data + b * stride_b + h * stride_h + s * stride_s;
    }
    __device__ __forceinline__ const half* get_ptr(int b, int h, int s, int d) const {
        return data + b * stride_b + h * stride_h + s * stride_s + d * stride_d;
    }
#endif
};

}  // namespace cuda
}  // namespace engine
