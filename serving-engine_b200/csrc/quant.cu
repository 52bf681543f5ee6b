// quant.cu -- FP8 (OCP E4M3) and 4-bit weight quantisation for the decode
// GEMVs.
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

// 4-bit weights (layout: kI4Group in gemv.cuh).  One warp per group of 128
// weights, 4 per lane: lane l holds weights 4l .. 4l + 3, i.e. half of the
// 32-bit word l / 2 of the group, which it assembles with its neighbour.
// Grid (groups of a row / 8, rows), 256 threads.
__global__ void __launch_bounds__(256) quant_i4_rows_kernel(const __half* __restrict__ w, int K,
                                                            uint8_t* __restrict__ q, float* __restrict__ scales) {
    griddep_wait();
    griddep_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int groups = K / kI4Group;
    const int g = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (g >= groups) return;
    const size_t row = blockIdx.y;
    const __half* src = w + row * K + (size_t)g * kI4Group + 4 * lane;
    const uint2 raw = *reinterpret_cast<const uint2*>(src);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
    const float v[4] = {a.x, a.y, b.x, b.y};
    float mx = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    mx = warp_max(mx);
    const float sc = mx / 7.0f;
    // weight j of a word (j = 4 (l & 1) + e here) sits at bit 16 (j & 1) + 4 (j >> 1)
    uint32_t bits = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int j = 4 * (lane & 1) + e;
        float qv = sc > 0.f ? rintf(v[e] / sc) : 0.f;
        qv = fminf(7.f, fmaxf(-7.f, qv));
        bits |= (uint32_t)((int)qv + 8) << (16 * (j & 1) + 4 * (j >> 1));
    }
    bits |= __shfl_xor_sync(0xffffffffu, bits, 1);
    if ((lane & 1) == 0)
        reinterpret_cast<uint32_t*>(q + row * (K / 2) + (size_t)g * (kI4Group / 2))[lane >> 1] = bits;
    if (lane == 0) scales[row * groups + g] = sc;
}

int quantize_i4_rows(const __half* w, int64_t rows, int K, uint8_t* q, float* scales, cudaStream_t s) {
    if (rows <= 0 || K <= 0) return B2_OK;
    if (K % kI4Group || !aligned16(w) || !aligned16(q)) return B2_ERR_UNSUPPORTED;
    const int groups = K / kI4Group;
    for (int64_t r0 = 0; r0 < rows; r0 += 65535) {
        const int64_t nr = rows - r0 < 65535 ? rows - r0 : 65535;
        B2_TRY(launch(quant_i4_rows_kernel, dim3((unsigned)((groups + 7) / 8), (unsigned)nr), dim3(256), 0, s, true,
                      w + r0 * K, K, q + r0 * (K / 2), scales + r0 * groups));
    }
    return B2_OK;
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

extern "C" int b2_quantize_int4_rows(const void* w, int64_t rows, int K, void* q, float* scales, void* stream) {
    using namespace b2;
    B2_REQUIRE(w && q && scales && rows >= 0 && K >= 0);
    return quantize_i4_rows(static_cast<const __half*>(w), rows, K, static_cast<uint8_t*>(q), scales,
                            as_stream(stream));
}

extern "C" int b2_gemv_int4(const void* Wq, const float* scales, const void* x, void* y, int B, int N, int K,
                            int out_f32, void* stream) {
    using namespace b2;
    if (N <= 0 || K <= 0 || B <= 0) return B2_OK;
    B2_REQUIRE(Wq && scales && x && y);
    if ((K % kI4Group) || !aligned16(Wq) || !aligned16(x)) return B2_ERR_UNSUPPORTED;
    for (int b0 = 0; b0 < B; b0 += 2) {
        const int nb = B - b0 < 2 ? B - b0 : 2;
        GemvParams p = {};
        p.W8 = static_cast<const uint8_t*>(Wq);
        p.w4 = 1;
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
