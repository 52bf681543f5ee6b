// skinny.cu -- Y = X W^T for decode batches: X is a handful of activation
// rows (the batch), W a projection's weight matrix read once per step.
//
// The weights take the MMA's M side (128 weight rows per tile) and the batch
// its N side (NB = 32, 64, 128 or 256 columns, rows of X beyond the batch
// zero-filled by TMA), so one tcgen05.mma (M=128, N=NB, K=16) covers the
// whole batch and the accumulator is NB fp32 columns of TMEM.  The kernel is
// a weight stream: one CTA per SM, a ring of 64-deep stages (16 KB of
// weights + NB x 64 of X) as deep as shared memory allows, and the flattened
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
#include "skinny.cuh"
#include "tc.cuh"

namespace b2 {

template <int NB>
struct SkCfg {
    static constexpr uint32_t W_BYTES = 128 * 64 * 2;
    static constexpr uint32_t X_BYTES = NB * 64 * 2;
    static constexpr uint32_t STAGE = W_BYTES + X_BYTES;
    static constexpr int STAGES = (200 * 1024) / STAGE > 12 ? 12 : (200 * 1024) / STAGE;
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

SkinnyPlan skinny_plan(int N, int K) {
    SkinnyPlan p;
    p.nk = (K + 63) / 64;
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

}  // namespace b2
