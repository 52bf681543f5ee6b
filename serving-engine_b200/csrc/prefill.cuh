// prefill.cuh -- arguments of the flash prefill (prefill.cu), shared with the
// model runtime.
#pragma once

#include "common.cuh"

namespace b2 {

struct FlashArgs {
    const void* q;
    const void* k;
    const void* v;
    void* out;
    int S, nq, nkv, D, batch;
    int64_t ldq, ldkv, ldo;  // elements between consecutive tokens
    bool bf16;
    float rope_theta;  // > 0: q and k rotated (positions pos0..) by a pre-pass
    int pos0;
    // RoPE form: device scratch for the rotated q and k copies
    // (batch*S*(nq+nkv)*D*2 bytes); null: the library's per-device buffer,
    // grown on demand
    void* rk_ws;
    size_t rk_ws_bytes;
};

int flash_prefill_tc(const FlashArgs& a, cudaStream_t s);
int causal_attention_rows_ld(const __half* q, int64_t ldq, const __half* k, const __half* v, int64_t ldkv,
                             __half* out, int64_t ldo, int64_t S, int nq, int nkv, int D, int batch, cudaStream_t s);

}  // namespace b2
