// ops.cu -- elementwise and row operators of the operator API
// (embedding, RMSNorm, bias / residual add, RoPE, SwiGLU, softmax, KV append).
//
// On the decode hot path these are fused into the GEMV prologues/epilogues
// (gemv.cu); the standalone forms here keep the reference operator API
// (src/cuda/kernels.h) for its callers and tests.
#include <cmath>

#include "common.cuh"

namespace b2 {

// ---------------------------------------------------------------------------
// embedding: one CTA per token row, 16-byte copies when rows are aligned.
// Reference: src/cuda/embedding.cu:7-41.
// ---------------------------------------------------------------------------
__global__ void embedding_kernel(const int64_t* __restrict__ ids, const __half* __restrict__ table,
                                 __half* __restrict__ out, int64_t hidden, int vec) {
    griddep_wait();
    const int64_t s = blockIdx.x;
    const int64_t id = ids[s];
    const __half* src = table + id * hidden;
    __half* dst = out + s * hidden;
    if (vec) {
        const int64_t n8 = hidden >> 3;
        for (int64_t i = threadIdx.x; i < n8; i += blockDim.x)
            reinterpret_cast<uint4*>(dst)[i] = ldg16(reinterpret_cast<const uint4*>(src) + i);
    } else {
        for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) dst[i] = src[i];
    }
}

// ---------------------------------------------------------------------------
// RMSNorm: one CTA per row, fp32 sum of squares, out = half(x * r * w).
// Reference: src/cuda/rmsnorm.cu:16-70, src/cpu/ops.cpp:26-51.
// ---------------------------------------------------------------------------
__global__ void rmsnorm_kernel(const __half* __restrict__ x, const __half* __restrict__ w,
                               __half* __restrict__ out, int64_t dim, float eps) {
    __shared__ float red[32];
    griddep_wait();
    const __half* xr = x + blockIdx.x * dim;
    __half* o = out + blockIdx.x * dim;
    float ss = 0.f;
    for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) {
        float v = __half2float(xr[i]);
        ss = fmaf(v, v, ss);
    }
    ss = block_sum(ss, red);
    const float r = rsqrtf(ss / (float)dim + eps);
    for (int64_t i = threadIdx.x; i < dim; i += blockDim.x)
        o[i] = __float2half_rn(__half2float(xr[i]) * r * __half2float(w[i]));
}

// Reference: src/cuda/bias_add.cu:7-22
__global__ void bias_add_kernel(const __half* __restrict__ x, const __half* __restrict__ b,
                                __half* __restrict__ out, int64_t M, int64_t N) {
    griddep_wait();
    const int64_t total = M * N;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = __float2half_rn(__half2float(x[i]) + __half2float(b[i % N]));
}

// Reference: src/cuda/residual_add.cu:7-19
__global__ void residual_add_kernel(const __half* __restrict__ a, const __half* __restrict__ b,
                                    __half* __restrict__ out, int64_t n) {
    griddep_wait();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = __float2half_rn(__half2float(a[i]) + __half2float(b[i]));
}

// ---------------------------------------------------------------------------
// RoPE (rotate-half) in place.  One thread per (token, head, pair i).
// Reference: src/cuda/rope.cu:8-58, src/cpu/ops.cpp:165-221.
// ---------------------------------------------------------------------------
__global__ void rope_kernel(__half* __restrict__ q, __half* __restrict__ k, int64_t S, int64_t nq,
                            int64_t nkv, int64_t D, int64_t start_pos, float theta) {
    griddep_wait();
    const int64_t half = D / 2;
    const int64_t heads = nq + nkv;
    const int64_t total = S * heads * half;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t % half;
        const int64_t h = (t / half) % heads;
        const int64_t s = t / (half * heads);
        const float inv = 1.0f / powf(theta, (float)(2 * i) / (float)D);
        const float a = (float)(start_pos + s) * inv;
        float sn, cs;
        sincosf(a, &sn, &cs);
        __half* v = h < nq ? q + (s * nq + h) * D : k + (s * nkv + (h - nq)) * D;
        const float x1 = __half2float(v[i]), x2 = __half2float(v[i + half]);
        v[i] = __float2half_rn(x1 * cs - x2 * sn);
        v[i + half] = __float2half_rn(x2 * cs + x1 * sn);
    }
}

// Reference: src/cuda/swiglu.cu:8-25 (silu(g) = g / (1 + exp(-g)))
__global__ void swiglu_kernel(const __half* __restrict__ g, const __half* __restrict__ u,
                              __half* __restrict__ out, int64_t n) {
    griddep_wait();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float gv = __half2float(g[i]);
        out[i] = __float2half_rn(gv / (1.0f + expf(-gv)) * __half2float(u[i]));
    }
}

// Reference: src/cuda/softmax.cu:25-83
__global__ void softmax_kernel(const __half* __restrict__ x, __half* __restrict__ out, int64_t cols) {
    __shared__ float red[32];
    griddep_wait();
    const __half* xr = x + blockIdx.x * cols;
    __half* o = out + blockIdx.x * cols;
    float m = -3.0e38f;
    for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) m = fmaxf(m, __half2float(xr[i]));
    m = block_max(m, red);
    float s = 0.f;
    for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) s += expf(__half2float(xr[i]) - m);
    s = block_sum(s, red);
    const float inv = 1.0f / s;
    for (int64_t i = threadIdx.x; i < cols; i += blockDim.x)
        o[i] = __float2half_rn(expf(__half2float(xr[i]) - m) * inv);
}

// ---------------------------------------------------------------------------
// KV append: token-major [T, nkv, D] -> head-major [nkv, max_seq, D].
// One thread per 8-element chunk (or per element when D % 8 != 0).
// Reference: src/runtime/kv_cache.cu:8-61.
// ---------------------------------------------------------------------------
__global__ void append_kv_kernel(const __half* __restrict__ sk, const __half* __restrict__ sv,
                                 __half* __restrict__ dk, __half* __restrict__ dv, int T, int p0,
                                 int nkv, int max_seq, int D, int vec) {
    griddep_wait();
    const int per = vec ? D / 8 : D;
    const int64_t total = (int64_t)T * nkv * per;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(t % per);
        const int h = (int)((t / per) % nkv);
        const int tok = (int)(t / ((int64_t)per * nkv));
        const int pos = p0 + tok;
        if (pos >= max_seq) continue;
        const int64_t so = ((int64_t)tok * nkv + h) * D;
        const int64_t dof = ((int64_t)h * max_seq + pos) * D;
        if (vec) {
            reinterpret_cast<uint4*>(dk + dof)[c] = reinterpret_cast<const uint4*>(sk + so)[c];
            reinterpret_cast<uint4*>(dv + dof)[c] = reinterpret_cast<const uint4*>(sv + so)[c];
        } else {
            dk[dof + c] = sk[so + c];
            dv[dof + c] = sv[so + c];
        }
    }
}

static inline unsigned grid_for(int64_t n, int threads) {
    int64_t g = (n + threads - 1) / threads;
    const int64_t cap = (int64_t)sm_count() * 16;
    if (g > cap) g = cap;
    return (unsigned)(g < 1 ? 1 : g);
}

}  // namespace b2

using namespace b2;

extern "C" int b2_embedding_lookup(const int64_t* ids, const void* table, void* out, int64_t seq_len,
                                   int64_t hidden, void* stream) {
    if (seq_len <= 0) return B2_OK;
    B2_REQUIRE(ids && table && out && hidden > 0);
    const int vec = (hidden % 8 == 0) && aligned16(table) && aligned16(out);
    const int threads = hidden >= 256 ? 256 : (int)((hidden + 31) / 32 * 32);
    B2_TRY(launch(embedding_kernel, dim3((unsigned)seq_len), dim3(threads), 0, as_stream(stream), true,
                  ids, (const __half*)table, (__half*)out, hidden, vec));
    return B2_OK;
}

extern "C" int b2_rmsnorm(const void* x, const void* w, void* out, int64_t rows, int64_t dim, float eps,
                          void* stream) {
    if (rows <= 0) return B2_OK;
    B2_REQUIRE(x && w && out && dim > 0);
    const int threads = dim >= 256 ? 256 : (int)((dim + 31) / 32 * 32);
    B2_TRY(launch(rmsnorm_kernel, dim3((unsigned)rows), dim3(threads), 0, as_stream(stream), true,
                  (const __half*)x, (const __half*)w, (__half*)out, dim, eps));
    return B2_OK;
}

extern "C" int b2_bias_add(const void* x, const void* b, void* out, int64_t M, int64_t N, void* stream) {
    if (M <= 0 || N <= 0) return B2_OK;
    B2_REQUIRE(x && b && out);
    B2_TRY(launch(bias_add_kernel, dim3(grid_for(M * N, 256)), dim3(256), 0, as_stream(stream), true,
                  (const __half*)x, (const __half*)b, (__half*)out, M, N));
    return B2_OK;
}

extern "C" int b2_residual_add(const void* a, const void* b, void* out, int64_t n, void* stream) {
    if (n <= 0) return B2_OK;
    B2_REQUIRE(a && b && out);
    B2_TRY(launch(residual_add_kernel, dim3(grid_for(n, 256)), dim3(256), 0, as_stream(stream), true,
                  (const __half*)a, (const __half*)b, (__half*)out, n));
    return B2_OK;
}

extern "C" int b2_apply_rope(void* q, void* k, int64_t S, int64_t nq, int64_t nkv, int64_t D,
                             int64_t start_pos, float theta, void* stream) {
    if (S <= 0) return B2_OK;
    B2_REQUIRE(q && k && D >= 2 && nq >= 0 && nkv >= 0);
    const int64_t total = S * (nq + nkv) * (D / 2);
    if (total == 0) return B2_OK;
    B2_TRY(launch(rope_kernel, dim3(grid_for(total, 256)), dim3(256), 0, as_stream(stream), true,
                  (__half*)q, (__half*)k, S, nq, nkv, D, start_pos, theta));
    return B2_OK;
}

extern "C" int b2_swiglu(const void* g, const void* u, void* out, int64_t n, void* stream) {
    if (n <= 0) return B2_OK;
    B2_REQUIRE(g && u && out);
    B2_TRY(launch(swiglu_kernel, dim3(grid_for(n, 256)), dim3(256), 0, as_stream(stream), true,
                  (const __half*)g, (const __half*)u, (__half*)out, n));
    return B2_OK;
}

extern "C" int b2_softmax(const void* x, void* out, int64_t rows, int64_t cols, void* stream) {
    if (rows <= 0 || cols <= 0) return B2_OK;
    B2_REQUIRE(x && out);
    const int threads = cols >= 256 ? 256 : (int)((cols + 31) / 32 * 32);
    B2_TRY(launch(softmax_kernel, dim3((unsigned)rows), dim3(threads), 0, as_stream(stream), true,
                  (const __half*)x, (__half*)out, cols));
    return B2_OK;
}

extern "C" int b2_append_kv_cache(const void* sk, const void* sv, void* dk, void* dv, int T, int p0,
                                  int nkv, int max_seq, int D, void* stream) {
    if (T <= 0) return B2_OK;
    B2_REQUIRE(sk && sv && dk && dv && nkv > 0 && D > 0 && max_seq > 0 && p0 >= 0);
    const int vec = (D % 8 == 0) && aligned16(sk) && aligned16(sv) && aligned16(dk) && aligned16(dv);
    const int64_t total = (int64_t)T * nkv * (vec ? D / 8 : D);
    B2_TRY(launch(append_kv_kernel, dim3(grid_for(total, 256)), dim3(256), 0, as_stream(stream), true,
                  (const __half*)sk, (const __half*)sv, (__half*)dk, (__half*)dv, T, p0, nkv, max_seq, D,
                  vec));
    return B2_OK;
}
