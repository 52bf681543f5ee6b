// prefill.cu -- causal GQA prefill attention (operator API flash_prefill_gqa).
//
// Current form: every query row is run as a decode query of length i+1
// through the split-KV attention kernel (attention.cu), which streams K/V
// once per kv head for the whole query-head group with online softmax.
// Reference replaced: src/cuda/flash_prefill.cu:43-240.
#include "common.cuh"

namespace b2 {
int causal_attention_rows(const __half* q, const __half* k, const __half* v, __half* out, int64_t S, int nq,
                          int nkv, int D, int batch, cudaStream_t s);
bool attn_head_dim_supported(int D);
}  // namespace b2

extern "C" int b2_flash_prefill_gqa(const void* q, const void* k, const void* v, void* out, int64_t S, int nq,
                                    int nkv, int D, int batch, void* stream) {
    using namespace b2;
    if (S <= 0 || batch <= 0) return B2_OK;
    B2_REQUIRE(q && k && v && out && nq > 0 && nkv > 0 && nq % nkv == 0);
    if (!attn_head_dim_supported(D) || !aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
        return B2_ERR_UNSUPPORTED;
    return causal_attention_rows((const __half*)q, (const __half*)k, (const __half*)v, (__half*)out, S, nq, nkv, D,
                                 batch, as_stream(stream));
}
