// gemv.cuh -- parameters of the decode GEMV family (shared by gemv.cu and the
// model runtime).
#pragma once

#include "common.cuh"

namespace b2 {

// How the activation vector x is produced in the CTA prologue.
enum XMode : int {
    X_HALF = 0,  // x is half [B, ldx] written by the previous kernel
    X_NORM = 1,  // x = half(h * rsqrt(mean(h^2) + eps) * norm_w), h float [B, ldx]
};

// What the epilogue does with the fp32 dot products of a warp task.
enum OutMode : int {
    OUT_HALF = 0,    // y half [B, ldy] (+bias / +residual)
    OUT_F32 = 1,     // y float [B, ldy] (+bias / +residual)
    OUT_RESID = 2,   // hidden float [B, ldy]: y = dot + (resid_add ? y : 0)
    OUT_QKV = 3,     // fused q|k|v rows, rotate-half RoPE, K/V into the cache
    OUT_SWIGLU = 4,  // act half [B, ldy] = silu(dot(Wg)) * dot(Wu)
    OUT_LOGITS = 5,  // logits float [B, ldy] and a packed argmax per sequence
};

struct GemvParams {
    const __half* W;   // [rows, K] row-major
    const __half* W2;  // OUT_SWIGLU: up-projection rows
    int K;
    int tasks;  // warp tasks: rows (R=1) or row pairs (R=2)
    int B;      // sequences in this launch (<= the batch tile)

    const void* x;  // half or float [B, ldx]
    int64_t ldx;
    const __half* norm_w;
    float eps;

    const __half* bias;   // [rows] or null
    const __half* resid;  // half residual [B, ld_resid] or null (OUT_HALF/OUT_F32)
    int64_t ld_resid;
    int resid_add;        // OUT_RESID: 1 adds the existing y (residual stream)
    void* y;
    int64_t ldy;

    // OUT_QKV
    int nq, nkv, D;
    const float2* rope;  // [max_pos, D/2] (cos, sin)
    const int* pos;      // [B] positions of the new token
    __half* kcache;      // this layer's K base: + b*kv_sb + h*kv_sh + pos*D
    __half* vcache;
    int64_t kv_sb, kv_sh;

    // OUT_LOGITS
    unsigned long long* argmax;  // [B] packed (value, id), 0 before the launch
    int row_offset;              // global id of local row 0 (vocabulary shard)
    int argmax_limit;            // global ids >= limit are not candidates
};

// Launch the vectorised GEMV.  Requires K % 8 == 0 and 16-byte aligned W,
// W2, x rows; returns B2_ERR_UNSUPPORTED otherwise.  B <= 8 per launch.
int gemv_launch(const GemvParams& p, XMode xm, OutMode om, cudaStream_t s, bool pdl);

// Maximum batch tile handled by one gemv_launch for row length K.
int gemv_batch_tile(int K);

}  // namespace b2
