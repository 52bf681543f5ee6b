// skinny.cuh -- decode-batch projections on the tensor cores (see skinny.cu).
#pragma once

#include "common.cuh"

namespace b2 {

// Work split of one skinny launch: the weight rows are cut into 128-row
// tiles, each tile into nk 64-deep k blocks, and the tiles * nk (tile, k
// block) iterations into equal consecutive ranges of `per`, one per CTA
// ("stream-K").  A CTA writes one fp32 partial per tile its range touches.
struct SkinnyPlan {
    int nk;         // k blocks per tile
    int per;        // iterations per CTA
    int ctas;       // grid size
    int max_slabs;  // most partials any tile gets
};

// Partials of output column n (weight row n of the concatenated weights):
// slabs 0 .. sk_nseg - 1 of ws[slab][batch][N], summed in slab order.
__host__ __device__ __forceinline__ int sk_nseg(int n, int nk, int per) {
    const int t = n >> 7;
    return (t * nk + nk - 1) / per - (t * nk) / per + 1;
}

// kdepth: elements of K per k block (64 for half weights, 128 for FP8).
SkinnyPlan skinny_plan(int N, int K, int kdepth = 64);

// ws[slab][b][n] partials of Y[b][n] = sum_k X[b][k] W[n][k] for b < B,
// W = W0 (rows 0..N0-1) followed by W1 (N1 rows; may be null with N1 = 0,
// else N0 % 128 == 0).  X [B][K] half, rows K apart; W row-major [rows][K].
// B <= 256, K % 8 == 0, 16-byte aligned bases.  ws must hold
// plan.max_slabs * B * (N0 + N1) floats (B2_ERR_INVALID otherwise).
// tr: the step trace's slot for this launch (buf null: off).
int gemm_skinny(const __half* X, int B, const __half* W0, int N0, const __half* W1, int N1, int K, float* ws,
                size_t ws_floats, SkinnyPlan* plan, cudaStream_t s, TraceSlot tr = TraceSlot{nullptr, 0});

// As gemm_skinny with FP8 (E4M3) weights: codes W0q [N0][K], W1q [N1][K]
// (bytes), one fp32 scale per row (sc0, sc1); ws receives the scaled
// partials, so the consumers are those of the half form.  128-deep k blocks
// (plan.nk = ceil(K / 128)); B <= 128, K % 16 == 0.
int gemm_skinny_f8(const __half* X, int B, const uint8_t* W0q, const float* sc0, int N0, const uint8_t* W1q,
                   const float* sc1, int N1, int K, float* ws, size_t ws_floats, SkinnyPlan* plan, cudaStream_t s,
                   TraceSlot tr = TraceSlot{nullptr, 0});

}  // namespace b2
