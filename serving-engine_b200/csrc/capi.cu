// capi.cu -- status strings, build identification, the bounded-wait error
// word of the tcgen05 kernels, and TMA tensor-map encoding.
#include <cudaTypedefs.h>

#include <mutex>

#include "tc.cuh"

namespace b2 {

// Set (first writer wins) by a tcgen05 kernel whose bounded mbarrier wait
// gave up; read and cleared by b2_device_status.
static __device__ int g_wait_error;

static std::mutex g_err_mu;
static int* g_err_ptr[64];

int* wait_error_word() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(g_err_mu);
    if (!g_err_ptr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_wait_error) != cudaSuccess) return nullptr;
        g_err_ptr[dev] = static_cast<int*>(p);
    }
    return g_err_ptr[dev];
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, []() {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

static int encode_map(CUtensorMap* map, CUtensorMapDataType type, int rank, const void* base, const uint64_t* dims,
                      const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz) {
    auto fn = encode_fn();
    if (!fn) return B2_ERR_UNSUPPORTED;
    cuuint64_t d[5], st[4];
    cuuint32_t bx[5], es[5];
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        bx[i] = box[i];
        es[i] = 1;
        if (i + 1 < rank) st[i] = strides_bytes[i];
    }
    const CUresult r = fn(map, type, (cuuint32_t)rank, const_cast<void*>(base), d, st, bx, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? B2_OK : B2_ERR_UNSUPPORTED;
}

int make_tensor_map(CUtensorMap* map, CUtensorMapDataType type, int rank, const void* base, const uint64_t* dims,
                    const uint64_t* strides_bytes, const uint32_t* box) {
    return encode_map(map, type, rank, base, dims, strides_bytes, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

int make_tensor_map_plain(CUtensorMap* map, CUtensorMapDataType type, int rank, const void* base,
                          const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box) {
    return encode_map(map, type, rank, base, dims, strides_bytes, box, CU_TENSOR_MAP_SWIZZLE_NONE);
}

}  // namespace b2

extern "C" const char* b2_version(void) { return "b2engine 0.1 sm_100a"; }

extern "C" const char* b2_status_string(int status) {
    switch (status) {
        case B2_OK: return "ok";
        case B2_ERR_INVALID: return "invalid argument";
        case B2_ERR_UNSUPPORTED: return "unsupported shape or alignment";
        case B2_ERR_WORKSPACE: return "workspace too small";
        case B2_ERR_NCCL: return "NCCL error";
        case B2_ERR_STATE: return "invalid state";
        case B2_ERR_TIMEOUT: return "device wait timed out";
        default:
            if (status > 0) return cudaGetErrorString(static_cast<cudaError_t>(status));
            return "unknown status";
    }
}

extern "C" int b2_device_status(int clear) {
    int* p = b2::wait_error_word();
    if (!p) return B2_ERR_STATE;
    int v = 0;
    B2_TRY(cudaDeviceSynchronize());
    B2_TRY(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost));
    if (clear && v) {
        const int zero = 0;
        B2_TRY(cudaMemcpy(p, &zero, sizeof(int), cudaMemcpyHostToDevice));
    }
    return v ? B2_ERR_TIMEOUT : B2_OK;
}
