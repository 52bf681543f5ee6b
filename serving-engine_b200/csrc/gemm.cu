// gemm.cu -- C = A * B^T for prefill projections (operator API
// matmul_transB / matmul_transB_f32).
//
// Shared-memory tiled CUDA-core kernel, fp32 accumulation: 64x64 output tile
// per CTA, 16-deep k slabs, 4x4 outputs per thread.  M = 1 goes to the decode
// GEMV.  Reference replaced: src/cuda/matmul.cu:23-79 (cublasGemmEx).
#include "common.cuh"

namespace b2 {

constexpr int TM = 64, TN = 64, TK = 16;

template <bool OUT_F32>
__global__ void __launch_bounds__(256) gemm_tn_kernel(const __half* __restrict__ A, const __half* __restrict__ B,
                                                      void* __restrict__ C, int M, int K, int N) {
    __shared__ float As[TK][TM + 4];
    __shared__ float Bs[TK][TN + 4];
    griddep_wait();
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += TK) {
        for (int i = threadIdx.x; i < TM * TK; i += 256) {
            const int r = i / TK, kk = i - (i / TK) * TK;
            const int gm = m0 + r, gk = k0 + kk;
            As[kk][r] = (gm < M && gk < K) ? __half2float(A[(size_t)gm * K + gk]) : 0.f;
            const int gn = n0 + r;
            Bs[kk][r] = (gn < N && gk < K) ? __half2float(B[(size_t)gn * K + gk]) : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < TK; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int gm = m0 + ty * 4 + i;
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int gn = n0 + tx * 4 + j;
            if (gn >= N) continue;
            if (OUT_F32) static_cast<float*>(C)[(size_t)gm * N + gn] = acc[i][j];
            else static_cast<__half*>(C)[(size_t)gm * N + gn] = __float2half_rn(acc[i][j]);
        }
    }
}

static int gemm_api(const void* A, const void* B, void* C, int M, int K, int N, bool f32, void* stream) {
    if (M <= 0 || N <= 0) return B2_OK;
    B2_REQUIRE(A && B && C && K >= 0);
    cudaStream_t s = as_stream(stream);
    if (M == 1 && K > 0) return b2_gemv_batched(B, A, nullptr, C, 1, N, K, 0, f32 ? 1 : 0, stream);
    dim3 grid((unsigned)((N + TN - 1) / TN), (unsigned)((M + TM - 1) / TM));
    if (f32)
        B2_TRY(launch(gemm_tn_kernel<true>, grid, dim3(256), 0, s, true, (const __half*)A, (const __half*)B, C, M, K, N));
    else
        B2_TRY(launch(gemm_tn_kernel<false>, grid, dim3(256), 0, s, true, (const __half*)A, (const __half*)B, C, M, K, N));
    return B2_OK;
}

}  // namespace b2

extern "C" int b2_matmul_transB(const void* A, const void* B, void* C, int M, int K, int N, void* stream) {
    return b2::gemm_api(A, B, C, M, K, N, false, stream);
}

extern "C" int b2_matmul_transB_f32(const void* A, const void* B, float* C, int M, int K, int N, void* stream) {
    return b2::gemm_api(A, B, C, M, K, N, true, stream);
}
