// skinny.cu -- Y = X W^T for decode batches: X is a handful of activation
// rows (the batch), W a projection's weight matrix read once per step.
//
// The weights take the MMA's M side (128 weight rows per tile) and the batch
// its N side (NB = 32, 64, 128 or 256 columns, rows of X beyond the batch
// zero-filled by TMA), so one tcgen05.mma (M=128, N=NB, K=16) covers the
// whole batch and the accumulator is NB fp32 columns of TMEM.  The kernel is
// a weight stream: one CTA per SM, a ring of 64-deep stages (16 KB of
// weights + NB x 64 of X; 5 stages at NB = 32, see SkCfg), and the flattened
// (tile, k block) iteration space cut into equal consecutive ranges, one per
// CTA ("stream-K"), so every SM streams the same number of weight bytes
// whatever the tile count.  A range crossing a tile boundary produces one
// fp32 partial per tile; partials go to slabs ws[slab][b][n] and are summed
// in slab order by the consumer kernel (deterministic).  Two TMEM
// accumulators let the epilogue of one tile overlap the next tile's MMAs.
//   warp 4      TMA producer (weight tiles of the first stages are issued
//               before the programmatic-launch wait: they do not depend on
//               the previous kernel);
//   warp 5      MMA issuer;
//   warps 0..3  epilogue: TMEM lane = weight row, column = batch row, so
//               each 32-column TMEM load gives 32 batch rows of 32
//               consecutive outputs, stored coalesced.
// Every mbarrier wait is bounded (tc.cuh).
// Reference replaced: the per-token projections of src/model/forward_gpu.cu
// (cublasGemmEx through src/cuda/matmul.cu:23-79) at batch > 1.
#include <cuda_fp8.h>

#include "skinny.cuh"
#include "tc.cuh"

namespace b2 {

template <int NB>
struct SkCfg {
    static constexpr uint32_t W_BYTES = 128 * 64 * 2;
    static constexpr uint32_t X_BYTES = NB * 64 * 2;
    static constexpr uint32_t STAGE = W_BYTES + X_BYTES;
    // NB = 32 (decode batches up to 32): 5 stages (100 KB).  Measured in the
    // batch-8 / 32 decode step against 10 stages (200 KB): 2083 / 7268 tok/s
    // against 1999 / 7102 -- the projections after the attention and the
    // slab-sum consumers start sooner beside a smaller ring, and the weight
    // stream keeps its rate (gate|up 42.2 us either way); 4 stages began to
    // slow the stream.
    static constexpr uint32_t BUDGET = NB <= 32 ? 104 * 1024 : 200 * 1024;
    static constexpr int STAGES = BUDGET / STAGE > 12 ? 12 : BUDGET / STAGE;
    static constexpr uint32_t TMEM_COLS = 2 * NB;  // two accumulators
    static constexpr size_t SMEM = (size_t)STAGES * STAGE + 256 + 1024;
};

template <int NB>
__global__ void __launch_bounds__(192, 1)
    skinny_kernel(const __grid_constant__ CUtensorMap tmW0, const __grid_constant__ CUtensorMap tmW1,
                  const __grid_constant__ CUtensorMap tmX, float* __restrict__ ws, int B, int N, int T0, int nk,
                  int per, int total, int* err, TraceSlot tr) {
    using Cfg = SkCfg<NB>;
    constexpr int STAGES = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;   // [2]
    uint64_t* acc_empty = acc_full + 2;    // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            tc::mbar_init(&acc_full[a], 1);
            tc::mbar_init(&acc_empty[a], 128);
        }
        tc::fence_barrier_init();
    }
    if (warp == 0) tc::tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    griddep_launch_dependents();

    const int c = blockIdx.x;
    const int it0 = c * per;
    const int it1 = min(total, it0 + per);

    if (warp == 4) {
        if (lane == 0) {
            auto load_w = [&](int it, int s) {
                const int t = it / nk, kb = it - (it / nk) * nk;
                uint8_t* st = smem + s * Cfg::STAGE;
                if (t < T0) tc::tma_load_2d(st, &tmW0, &full[s], kb * 64, t * 128);
                else tc::tma_load_2d(st, &tmW1, &full[s], kb * 64, (t - T0) * 128);
            };
            auto load_x = [&](int it, int s) {
                const int kb = it - (it / nk) * nk;
                tc::tma_load_2d(smem + s * Cfg::STAGE + Cfg::W_BYTES, &tmX, &full[s], kb * 64, 0);
            };
            const int npre = min(STAGES, it1 - it0);
            for (int i = 0; i < npre; ++i) {
                tc::mbar_arrive_expect_tx(&full[i], Cfg::STAGE);
                load_w(it0 + i, i);
            }
            griddep_wait();  // X is the previous kernel's output
            for (int i = 0; i < npre; ++i) load_x(it0 + i, i);
            for (int i = npre; it0 + i < it1; ++i) {
                const int s = i % STAGES;
                const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
                if (!tc::mbar_wait(&empty[s], ph ^ 1u, err, 41)) break;
                tc::mbar_arrive_expect_tx(&full[s], Cfg::STAGE);
                load_w(it0 + i, s);
                load_x(it0 + i, s);
            }
        }
    } else if (warp == 5) {
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_f16(128, NB, false, false);
            int seg = 0;
            for (int i = 0; it0 + i < it1; ++i) {
                const int it = it0 + i;
                const int kb = it - (it / nk) * nk;
                const bool first = (i == 0) || kb == 0;
                const uint32_t acc = (uint32_t)(seg & 1);
                if (first && seg >= 2) {
                    if (!tc::mbar_wait(&acc_empty[acc], (uint32_t)((seg >> 1) - 1) & 1u, err, 42)) break;
                    tc::fence_after_sync();
                }
                const int s = i % STAGES;
                if (!tc::mbar_wait(&full[s], (uint32_t)(i / STAGES) & 1u, err, 43)) break;
                tc::fence_after_sync();
                const uint32_t a = tc::smem_u32(smem + s * Cfg::STAGE);
                const uint32_t b = a + Cfg::W_BYTES;
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    tc::mma_f16(tmem + acc * NB, tc::desc_k_sw128(a + 32 * k), tc::desc_k_sw128(b + 32 * k), idesc,
                                (first && k == 0) ? 0u : 1u);
                tc::mma_commit(&empty[s]);
                if (it == it1 - 1 || kb == nk - 1) {
                    tc::mma_commit(&acc_full[acc]);
                    ++seg;
                }
            }
        }
    } else {
        griddep_wait();  // ws may still be read by the previous kernel
        trace_begin(tr);
        const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
        int seg = 0;
        for (int it = it0; it < it1; ++seg) {
            const int t = it / nk;
            const int seg_end = min(it1, (t + 1) * nk);
            const uint32_t acc = (uint32_t)(seg & 1);
            const bool ok = __all_sync(0xffffffffu, tc::mbar_wait(&acc_full[acc], (uint32_t)(seg >> 1) & 1u, err, 44));
            if (!ok) break;
            tc::fence_after_sync();
            const int slab = c - (t * nk) / per;
            const int n = t * 128 + warp * 32 + lane;
            float* dst = ws + (size_t)slab * B * N + n;
#pragma unroll 1
            for (int cb = 0; cb < NB; cb += 32) {
                uint32_t v[32];
                tc::tmem_ld32(tmem + lane_base + acc * NB + cb, v);
                tc::tmem_wait_ld();
                if (n < N) {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (cb + j < B) dst[(size_t)(cb + j) * N] = __uint_as_float(v[j]);
                }
            }
            tc::fence_before_sync();
            tc::mbar_arrive(&acc_empty[acc]);
            it = seg_end;
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, Cfg::TMEM_COLS);
    }
    trace_end(tr);
}

// ---------------------------------------------------------------------------
// FP8 weights.  A stage holds a 128-row x 128-code tile of E4M3 weights
// (128-byte swizzled rows) and the matching 128 columns of X (two 64-column
// half atoms), each half with its own barrier: the weight tiles of the first
// stages are requested before the programmatic-launch wait and can be
// decoded before X arrives.  Four converter warps (warps 6..9, TMEM lane
// quarter w % 4) decode each weight row to halves (exact) into one of four
// TMEM staging buffers (64 columns: 128 halves in pairs); the MMA reads A
// from TMEM (tcgen05.mma ... [a_tmem], b_desc) and B = X from shared memory.
// The epilogue multiplies each row by its scale before writing the partial,
// so the slabs hold what the half form writes.
// ---------------------------------------------------------------------------
template <int NB>
struct SkF8Cfg {
    static constexpr uint32_t W_BYTES = 128 * 128;
    static constexpr uint32_t X_ATOM = NB * 128;  // NB rows x 64 halves
    static constexpr uint32_t STAGE = W_BYTES + 2 * X_ATOM;
    // NB = 32: 6 stages (147 KB); measured 2299 / 8007 tok/s at batch 8 / 32
    // against 2263 / 7807 with 8 (5 stages: 2289 / 7991)
    static constexpr uint32_t BUDGET = NB <= 32 ? 148 * 1024 : 200 * 1024;
    static constexpr int STAGES = BUDGET / STAGE > 8 ? 8 : BUDGET / STAGE;
    static constexpr int NA = 4;                   // TMEM staging buffers of decoded weights
    static constexpr uint32_t COL_A = 2 * NB;      // after the two accumulators, 64 columns each
    static constexpr uint32_t TMEM_COLS = 2 * NB + 64 * NA <= 256 ? 256 : 512;
    static constexpr size_t SMEM = (size_t)STAGES * STAGE + 512 + 1024;  // barriers: (3 STAGES + 4 + 2 NA) x 8 B
    static constexpr int THREADS = 320;
};

template <int NB>
__global__ void __launch_bounds__(320, 1)
    skinny_f8_kernel(const __grid_constant__ CUtensorMap tmW0, const __grid_constant__ CUtensorMap tmW1,
                     const __grid_constant__ CUtensorMap tmX, const float* __restrict__ sc0,
                     const float* __restrict__ sc1, int N0, float* __restrict__ ws, int B, int N, int T0, int nk,
                     int per, int total, int* err, TraceSlot tr) {
    using Cfg = SkF8Cfg<NB>;
    constexpr int STAGES = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE);  // X of stage s landed
    uint64_t* w_full = full + STAGES;      // weight codes of stage s landed
    uint64_t* empty = w_full + STAGES;
    uint64_t* acc_full = empty + STAGES;   // [2]
    uint64_t* acc_empty = acc_full + 2;    // [2]
    uint64_t* a_full = acc_empty + 2;      // [NA] decoded weights in TMEM buffer a
    uint64_t* a_empty = a_full + Cfg::NA;  // [NA]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(a_empty + Cfg::NA);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&w_full[s], 1);
            tc::mbar_init(&empty[s], 1 + 4);  // the MMA (X) and the four converter warps (weights)
        }
        for (int a = 0; a < 2; ++a) {
            tc::mbar_init(&acc_full[a], 1);
            tc::mbar_init(&acc_empty[a], 128);
        }
        for (int a = 0; a < Cfg::NA; ++a) {
            tc::mbar_init(&a_full[a], 4);
            tc::mbar_init(&a_empty[a], 1);
        }
        tc::fence_barrier_init();
    }
    if (warp == 0) tc::tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    griddep_launch_dependents();

    const int c = blockIdx.x;
    const int it0 = c * per;
    const int it1 = min(total, it0 + per);

    if (warp == 4) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            auto load_w = [&](int it, int s) {
                const int t = it / nk, kb = it - (it / nk) * nk;
                uint8_t* st = smem + s * Cfg::STAGE;
                tc::mbar_arrive_expect_tx(&w_full[s], Cfg::W_BYTES);
                if (t < T0) tc::tma_load_2d(st, &tmW0, &w_full[s], kb * 128, t * 128);
                else tc::tma_load_2d(st, &tmW1, &w_full[s], kb * 128, (t - T0) * 128);
            };
            auto load_x = [&](int it, int s) {
                const int kb = it - (it / nk) * nk;
                uint8_t* st = smem + s * Cfg::STAGE + Cfg::W_BYTES;
                tc::mbar_arrive_expect_tx(&full[s], 2 * Cfg::X_ATOM);
                tc::tma_load_2d(st, &tmX, &full[s], kb * 128, 0);
                tc::tma_load_2d(st + Cfg::X_ATOM, &tmX, &full[s], kb * 128 + 64, 0);
            };
            const int npre = min(STAGES, it1 - it0);
            for (int i = 0; i < npre; ++i) load_w(it0 + i, i);
            griddep_wait();  // X is the previous kernel's output
            for (int i = 0; i < npre; ++i) load_x(it0 + i, i);
            for (int i = npre; it0 + i < it1; ++i) {
                const int s = i % STAGES;
                const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
                if (!tc::mbar_wait(&empty[s], ph ^ 1u, err, 51)) break;
                load_w(it0 + i, s);
                load_x(it0 + i, s);
            }
        }
    } else if (warp >= 6) {
        // ---------------- E4M3 -> half converters: one weight row per thread ----------------
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        const int r = q * 32 + lane;
        const uint32_t lane_base = (uint32_t)(q * 32) << 16;
        for (int i = 0; it0 + i < it1; ++i) {
            const int s = i % STAGES, a = i % Cfg::NA;
            bool ok = __all_sync(0xffffffffu, tc::mbar_wait(&w_full[s], (uint32_t)(i / STAGES) & 1u, err, 52));
            if (ok && i >= Cfg::NA)
                ok = __all_sync(0xffffffffu,
                                tc::mbar_wait(&a_empty[a], (uint32_t)((i / Cfg::NA) - 1) & 1u, err, 53));
            if (!ok) break;
            tc::fence_after_sync();
            const uint8_t* row = smem + s * Cfg::STAGE + r * 128;
            uint32_t h[64];
#pragma unroll
            for (int j = 0; j < 8; ++j) {  // 16-byte chunk j of the row (128-byte swizzle)
                const uint4 w = *reinterpret_cast<const uint4*>(row + ((j ^ (r & 7)) << 4));
                const uint32_t ws4[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int m = 0; m < 4; ++m) {
                    const __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(ws4[m] & 0xffffu), __NV_E4M3);
                    const __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(ws4[m] >> 16), __NV_E4M3);
                    h[8 * j + 2 * m] = (uint32_t)lo.x | ((uint32_t)lo.y << 16);
                    h[8 * j + 2 * m + 1] = (uint32_t)hi.x | ((uint32_t)hi.y << 16);
                }
            }
            const uint32_t dst = tmem + lane_base + Cfg::COL_A + (uint32_t)a * 64;
            tc::tmem_st32(dst, *reinterpret_cast<uint32_t(*)[32]>(&h[0]));
            tc::tmem_st32(dst + 32, *reinterpret_cast<uint32_t(*)[32]>(&h[32]));
            tc::tmem_wait_st();
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) {
                tc::mbar_arrive(&a_full[a]);
                tc::mbar_arrive(&empty[s]);  // this stage's weight codes are consumed
            }
        }
    } else if (warp == 5) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_f16(128, NB, false, false);
            int seg = 0;
            for (int i = 0; it0 + i < it1; ++i) {
                const int it = it0 + i;
                const int kb = it - (it / nk) * nk;
                const bool first = (i == 0) || kb == 0;
                const uint32_t acc = (uint32_t)(seg & 1);
                if (first && seg >= 2) {
                    if (!tc::mbar_wait(&acc_empty[acc], (uint32_t)((seg >> 1) - 1) & 1u, err, 54)) break;
                    tc::fence_after_sync();
                }
                const int s = i % STAGES, a = i % Cfg::NA;
                if (!tc::mbar_wait(&full[s], (uint32_t)(i / STAGES) & 1u, err, 55)) break;
                if (!tc::mbar_wait(&a_full[a], (uint32_t)(i / Cfg::NA) & 1u, err, 56)) break;
                tc::fence_after_sync();
                const uint32_t xb = tc::smem_u32(smem + s * Cfg::STAGE + Cfg::W_BYTES);
                const uint32_t ab = tmem + Cfg::COL_A + (uint32_t)a * 64;
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    tc::mma_f16_ts(tmem + acc * NB, ab + (uint32_t)kk * 8,
                                   tc::desc_k_sw128(xb + (uint32_t)(kk >> 2) * Cfg::X_ATOM + (uint32_t)(kk & 3) * 32),
                                   idesc, (first && kk == 0) ? 0u : 1u);
                tc::mma_commit(&empty[s]);
                tc::mma_commit(&a_empty[a]);
                if (it == it1 - 1 || kb == nk - 1) {
                    tc::mma_commit(&acc_full[acc]);
                    ++seg;
                }
            }
        }
    } else {
        // ---------------- epilogue: scaled partials into the slabs ----------------
        griddep_wait();  // ws may still be read by the previous kernel
        trace_begin(tr);
        const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
        int seg = 0;
        for (int it = it0; it < it1; ++seg) {
            const int t = it / nk;
            const int seg_end = min(it1, (t + 1) * nk);
            const uint32_t acc = (uint32_t)(seg & 1);
            const bool ok = __all_sync(0xffffffffu, tc::mbar_wait(&acc_full[acc], (uint32_t)(seg >> 1) & 1u, err, 57));
            if (!ok) break;
            tc::fence_after_sync();
            const int slab = c - (t * nk) / per;
            const int n = t * 128 + warp * 32 + lane;
            const float scale = n < N ? (n < N0 ? sc0[n] : sc1[n - N0]) : 0.f;
            float* dst = ws + (size_t)slab * B * N + n;
#pragma unroll 1
            for (int cb = 0; cb < NB; cb += 32) {
                uint32_t v[32];
                tc::tmem_ld32(tmem + lane_base + acc * NB + cb, v);
                tc::tmem_wait_ld();
                if (n < N) {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (cb + j < B) dst[(size_t)(cb + j) * N] = __uint_as_float(v[j]) * scale;
                }
            }
            tc::fence_before_sync();
            tc::mbar_arrive(&acc_empty[acc]);
            it = seg_end;
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, Cfg::TMEM_COLS);
    }
    trace_end(tr);
}

SkinnyPlan skinny_plan(int N, int K, int kdepth) {
    SkinnyPlan p;
    p.nk = (K + kdepth - 1) / kdepth;
    const int tiles = (N + 127) / 128;
    const long total = (long)tiles * p.nk;
    const long g = sm_count();
    p.per = (int)((total + g - 1) / g);
    p.ctas = (int)((total + p.per - 1) / p.per);
    p.max_slabs = 0;
    for (int t = 0; t < tiles; ++t) {
        const int ns = sk_nseg(t * 128, p.nk, p.per);
        if (ns > p.max_slabs) p.max_slabs = ns;
    }
    return p;
}

template <int NB>
static int launch_skinny(const CUtensorMap& w0, const CUtensorMap& w1, const __half* X, int B, int N, int T0, int K,
                         float* ws, const SkinnyPlan& pl, int* err, cudaStream_t s, TraceSlot tr) {
    using Cfg = SkCfg<NB>;
    CUtensorMap tx;
    const uint64_t dx[2] = {(uint64_t)K, (uint64_t)B}, sx[1] = {(uint64_t)K * 2};
    const uint32_t bx[2] = {64u, (uint32_t)NB};
    const int rc = make_tensor_map(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, X, dx, sx, bx);
    if (rc != B2_OK) return rc;
    auto kern = skinny_kernel<NB>;
    B2_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg::SMEM));
    const int total = ((N + 127) / 128) * pl.nk;
    B2_TRY(launch(kern, dim3((unsigned)pl.ctas), dim3(192), Cfg::SMEM, s, true, w0, w1, tx, ws, B, N, T0, pl.nk,
                  pl.per, total, err, tr));
    return B2_OK;
}

int gemm_skinny(const __half* X, int B, const __half* W0, int N0, const __half* W1, int N1, int K, float* ws,
                size_t ws_floats, SkinnyPlan* plan, cudaStream_t s, TraceSlot tr) {
    if (B < 1 || B > 256 || N0 < 1 || K < 8 || (K & 7) || N1 < 0 || (N1 > 0 && (!W1 || (N0 & 127)))) return B2_ERR_INVALID;
    if (!aligned16(X) || !aligned16(W0) || (W1 && !aligned16(W1))) return B2_ERR_UNSUPPORTED;
    int* err = wait_error_word();
    if (!err) return B2_ERR_STATE;
    const int N = N0 + N1;
    const SkinnyPlan pl = skinny_plan(N, K);
    if ((size_t)pl.max_slabs * B * N > ws_floats) return B2_ERR_INVALID;
    if (plan) *plan = pl;
    CUtensorMap w0, w1;
    const uint32_t bw[2] = {64u, 128u};
    {
        const uint64_t d[2] = {(uint64_t)K, (uint64_t)N0}, st[1] = {(uint64_t)K * 2};
        const int rc = make_tensor_map(&w0, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, W0, d, st, bw);
        if (rc != B2_OK) return rc;
    }
    if (N1 > 0) {
        const uint64_t d[2] = {(uint64_t)K, (uint64_t)N1}, st[1] = {(uint64_t)K * 2};
        const int rc = make_tensor_map(&w1, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, W1, d, st, bw);
        if (rc != B2_OK) return rc;
    } else {
        w1 = w0;
    }
    const int T0 = N1 > 0 ? N0 / 128 : (N0 + 127) / 128;
    if (B <= 32) return launch_skinny<32>(w0, w1, X, B, N, T0, K, ws, pl, err, s, tr);
    if (B <= 64) return launch_skinny<64>(w0, w1, X, B, N, T0, K, ws, pl, err, s, tr);
    if (B <= 128) return launch_skinny<128>(w0, w1, X, B, N, T0, K, ws, pl, err, s, tr);
    return launch_skinny<256>(w0, w1, X, B, N, T0, K, ws, pl, err, s, tr);
}

template <int NB>
static int launch_skinny_f8(const CUtensorMap& w0, const CUtensorMap& w1, const __half* X, const float* sc0,
                            const float* sc1, int N0, int B, int N, int T0, int K, float* ws, const SkinnyPlan& pl,
                            int* err, cudaStream_t s, TraceSlot tr) {
    using Cfg = SkF8Cfg<NB>;
    CUtensorMap tx;
    const uint64_t dx[2] = {(uint64_t)K, (uint64_t)B}, sx[1] = {(uint64_t)K * 2};
    const uint32_t bx[2] = {64u, (uint32_t)NB};
    const int rc = make_tensor_map(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, X, dx, sx, bx);
    if (rc != B2_OK) return rc;
    auto kern = skinny_f8_kernel<NB>;
    B2_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg::SMEM));
    const int total = ((N + 127) / 128) * pl.nk;
    B2_TRY(launch(kern, dim3((unsigned)pl.ctas), dim3(Cfg::THREADS), Cfg::SMEM, s, true, w0, w1, tx, sc0, sc1, N0,
                  ws, B, N, T0, pl.nk, pl.per, total, err, tr));
    return B2_OK;
}

int gemm_skinny_f8(const __half* X, int B, const uint8_t* W0q, const float* sc0, int N0, const uint8_t* W1q,
                   const float* sc1, int N1, int K, float* ws, size_t ws_floats, SkinnyPlan* plan, cudaStream_t s,
                   TraceSlot tr) {
    if (B < 1 || B > 128 || N0 < 1 || K < 16 || (K & 15) || N1 < 0 || !sc0 ||
        (N1 > 0 && (!W1q || !sc1 || (N0 & 127))))
        return B2_ERR_INVALID;
    if (!aligned16(X) || !aligned16(W0q) || (W1q && !aligned16(W1q))) return B2_ERR_UNSUPPORTED;
    int* err = wait_error_word();
    if (!err) return B2_ERR_STATE;
    const int N = N0 + N1;
    const SkinnyPlan pl = skinny_plan(N, K, 128);
    if ((size_t)pl.max_slabs * B * N > ws_floats) return B2_ERR_INVALID;
    if (plan) *plan = pl;
    CUtensorMap w0, w1;
    const uint32_t bw[2] = {128u, 128u};
    {
        const uint64_t d[2] = {(uint64_t)K, (uint64_t)N0}, st[1] = {(uint64_t)K};
        const int rc = make_tensor_map(&w0, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, W0q, d, st, bw);
        if (rc != B2_OK) return rc;
    }
    if (N1 > 0) {
        const uint64_t d[2] = {(uint64_t)K, (uint64_t)N1}, st[1] = {(uint64_t)K};
        const int rc = make_tensor_map(&w1, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, W1q, d, st, bw);
        if (rc != B2_OK) return rc;
    } else {
        w1 = w0;
    }
    const int T0 = N1 > 0 ? N0 / 128 : (N0 + 127) / 128;
    if (B <= 32) return launch_skinny_f8<32>(w0, w1, X, sc0, sc1, N0, B, N, T0, K, ws, pl, err, s, tr);
    if (B <= 64) return launch_skinny_f8<64>(w0, w1, X, sc0, sc1, N0, B, N, T0, K, ws, pl, err, s, tr);
    return launch_skinny_f8<128>(w0, w1, X, sc0, sc1, N0, B, N, T0, K, ws, pl, err, s, tr);
}

}  // namespace b2
