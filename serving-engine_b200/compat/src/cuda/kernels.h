// compat/src/cuda/kernels.h -- the reference's operator API
// (src/cuda/kernels.h:14-219, namespace engine::cuda, void returns, errors as
// std::runtime_error) as inline forwarding wrappers over the b2engine C-ABI
// (include/b2engine.h).  Callers of the reference build unchanged against this
// header and link libb2engine.so; no reference kernel is compiled.
#pragma once

#include <cublas_v2.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "src/b2_compat.h"
#include "src/cuda/kv_view.h"

namespace engine {
namespace cuda {

inline b2_kv_view to_b2(const KVView& v) { return b2_kv_view{v.data, v.stride_b, v.stride_h, v.stride_s, v.stride_d}; }

inline void embedding_lookup(const int64_t* token_ids, const half* table, half* out, int64_t seq_len,
                             int64_t hidden_size, cudaStream_t stream = 0) {
    b2_check(b2_embedding_lookup(token_ids, table, out, seq_len, hidden_size, stream), "embedding_lookup");
}

inline void rmsnorm(const half* x, const half* weight, half* out, int64_t rows, int64_t dim, float eps = 1e-6f,
                    cudaStream_t stream = 0) {
    b2_check(b2_rmsnorm(x, weight, out, rows, dim, eps, stream), "rmsnorm");
}

inline void bias_add(const half* x, const half* bias, half* out, int64_t M, int64_t N, cudaStream_t stream = 0) {
    b2_check(b2_bias_add(x, bias, out, M, N, stream), "bias_add");
}

inline void residual_add(const half* a, const half* b, half* out, int64_t count, cudaStream_t stream = 0) {
    b2_check(b2_residual_add(a, b, out, count, stream), "residual_add");
}

inline void apply_rope(half* q, half* k, int64_t seq_len, int64_t num_q_heads, int64_t num_kv_heads,
                       int64_t head_dim, int64_t start_pos = 0, float rope_theta = 1000000.0f,
                       cudaStream_t stream = 0) {
    b2_check(b2_apply_rope(q, k, seq_len, num_q_heads, num_kv_heads, head_dim, start_pos, rope_theta, stream),
             "apply_rope");
}

inline void causal_gqa(const half* q, const half* k, const half* v, half* out, int64_t seq_len,
                       int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim, cudaStream_t stream = 0) {
    b2_check(b2_causal_gqa(q, k, v, out, seq_len, num_q_heads, num_kv_heads, head_dim, stream), "causal_gqa");
}

inline void softmax(const half* x, half* out, int64_t rows, int64_t cols, cudaStream_t stream = 0) {
    b2_check(b2_softmax(x, out, rows, cols, stream), "softmax");
}

inline void decode_gqa(const half* q, const half* k_cache, const half* v_cache, half* out, int total_seq_len,
                       int num_q_heads, int num_kv_heads, int max_seq, int head_dim, cudaStream_t stream = 0) {
    b2_check(b2_decode_gqa(q, k_cache, v_cache, out, total_seq_len, num_q_heads, num_kv_heads, max_seq, head_dim,
                           stream),
             "decode_gqa");
}

// The reference passes no buffer size; its callers allocate at least
// 8 * batch * heads * (head_dim + 2) floats (tests, bench, model), so that is
// what this wrapper promises the library.
inline void decode_gqa_split(const half* q, KVView k_view, KVView v_view, const int* seq_lens, half* out,
                             int batch_size, int num_q_heads, int num_kv_heads, int head_dim, int max_seq_len,
                             float* split_buffer = nullptr, cudaStream_t stream = 0) {
    const size_t floats = split_buffer ? (size_t)8 * batch_size * num_q_heads * (head_dim + 2) : 0;
    b2_check(b2_decode_gqa_split(q, to_b2(k_view), to_b2(v_view), seq_lens, out, batch_size, num_q_heads,
                                 num_kv_heads, head_dim, max_seq_len, split_buffer, floats, stream),
             "decode_gqa_split");
}

inline void flash_prefill_gqa(const half* q, const half* k, const half* v, half* out, int64_t seq_len,
                              int num_q_heads, int num_kv_heads, int head_dim, int batch_size = 1,
                              cudaStream_t stream = 0) {
    b2_check(b2_flash_prefill_gqa(q, k, v, out, seq_len, num_q_heads, num_kv_heads, head_dim, batch_size, stream),
             "flash_prefill_gqa");
}

inline void swiglu(const half* gate, const half* up, half* out, int64_t count, cudaStream_t stream = 0) {
    b2_check(b2_swiglu(gate, up, out, count, stream), "swiglu");
}

// The cuBLAS handle is accepted for signature compatibility and not used:
// the product runs on b2engine's tcgen05 GEMM (legacy default stream, like
// the reference's handle without a stream set).
inline void matmul_transB(cublasHandle_t /*handle*/, const half* A, const half* B, half* C, int M, int K, int N) {
    b2_check(b2_matmul_transB(A, B, C, M, K, N, nullptr), "matmul_transB");
}

inline void matmul_transB_f32(cublasHandle_t /*handle*/, const half* A, const half* B, float* C, int M, int K,
                              int N) {
    b2_check(b2_matmul_transB_f32(A, B, C, M, K, N, nullptr), "matmul_transB_f32");
}

inline void gemv(const half* W, const half* x, half* y, int N, int K, cudaStream_t stream = 0) {
    b2_check(b2_gemv(W, x, y, N, K, stream), "gemv");
}

inline void gemv_bias(const half* W, const half* x, const half* b, half* y, int N, int K, cudaStream_t stream = 0) {
    b2_check(b2_gemv_bias(W, x, b, y, N, K, stream), "gemv_bias");
}

inline void gemv_residual(const half* W, const half* x, const half* r, half* y, int N, int K,
                          cudaStream_t stream = 0) {
    b2_check(b2_gemv_residual(W, x, r, y, N, K, stream), "gemv_residual");
}

}  // namespace cuda
}  // namespace engine
