// quant.cu -- FP8 (OCP E4M3) weight quantisation for the decode GEMVs.
//
// Decode at batch 1-2 streams every weight byte once per token, so 1-byte
// weights halve the step's HBM traffic.  Format: per output row r of a
// [rows][K] fp16 matrix, scale_r = max_k |w[r][k]| / 448 (448 = largest
// finite E4M3 value; scale 1 for an all-zero row) and
// q[r][k] = E4M3(w[r][k] / scale_r) rounded to nearest even, saturating at
// +-448.  The GEMV decodes the codes to halves (every E4M3 value is exactly
// a half), accumulates sum_k q x in fp32 and multiplies by scale_r.  The
// reference has no quantised path (its RESULTS.md:39-40 plans INT8/INT4
// weights and FP8/INT8 KV as P8/P9).
#include <cuda_fp8.h>

#include "gemv.cuh"

namespace b2 {

constexpr float kE4M3Max = 448.0f;

// One CTA per row: the row's |w| maximum (exact in any order), then the codes.
__global__ void __launch_bounds__(256) quant_e4m3_rows_kernel(const __half* __restrict__ w, int K,
                                                              uint8_t* __restrict__ q, float* __restrict__ scales) {
    __shared__ float red[8];
    __shared__ float s_scale;
    griddep_wait();
    griddep_launch_dependents();
    const __half* row = w + (size_t)blockIdx.x * K;
    uint8_t* qr = q + (size_t)blockIdx.x * K;
    float mx = 0.f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) mx = fmaxf(mx, fabsf(__half2float(row[k])));
    mx = warp_max(mx);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x == 0) {
        float m = 0.f;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) m = fmaxf(m, red[i]);
        const float sc = m > 0.f ? m / kE4M3Max : 1.0f;
        s_scale = sc;
        scales[blockIdx.x] = sc;
    }
    __syncthreads();
    const float sc = s_scale;
    for (int k = threadIdx.x; k < K; k += blockDim.x)
        qr[k] = (uint8_t)__nv_cvt_float_to_fp8(__half2float(row[k]) / sc, __NV_SATFINITE, __NV_E4M3);
}

int quantize_e4m3_rows(const __half* w, int64_t rows, int K, uint8_t* q, float* scales, cudaStream_t s) {
    if (rows <= 0 || K <= 0) return B2_OK;
    if (rows > 0x7fffffff) return B2_ERR_UNSUPPORTED;
    B2_TRY(launch(quant_e4m3_rows_kernel, dim3((unsigned)rows), dim3(256), 0, s, true, w, K, q, scales));
    return B2_OK;
}

}  // namespace b2

extern "C" int b2_quantize_fp8_rows(const void* w, int64_t rows, int K, void* q, float* scales, void* stream) {
    using namespace b2;
    B2_REQUIRE(w && q && scales && rows >= 0 && K >= 0);
    return quantize_e4m3_rows(static_cast<const __half*>(w), rows, K, static_cast<uint8_t*>(q), scales,
                              as_stream(stream));
}

extern "C" int b2_gemv_fp8(const void* Wq, const float* scales, const void* x, void* y, int B, int N, int K,
                           int out_f32, void* stream) {
    using namespace b2;
    if (N <= 0 || K <= 0 || B <= 0) return B2_OK;
    B2_REQUIRE(Wq && scales && x && y);
    if ((K & 15) || !aligned16(Wq) || !aligned16(x)) return B2_ERR_UNSUPPORTED;
    const int bt = gemv_batch_tile(K);
    for (int b0 = 0; b0 < B; b0 += bt) {
        const int nb = B - b0 < bt ? B - b0 : bt;
        GemvParams p = {};
        p.W8 = static_cast<const uint8_t*>(Wq);
        p.wsc = scales;
        p.K = K;
        p.tasks = N;
        p.B = nb;
        p.x = static_cast<const __half*>(x) + (size_t)b0 * K;
        p.ldx = K;
        p.y = out_f32 ? (void*)(static_cast<float*>(y) + (size_t)b0 * N) : (void*)(static_cast<__half*>(y) + (size_t)b0 * N);
        p.ldy = N;
        const int rc = gemv_launch(p, X_HALF, out_f32 ? OUT_F32 : OUT_HALF, as_stream(stream), true);
        if (rc != B2_OK) return rc;
    }
    return B2_OK;
}
