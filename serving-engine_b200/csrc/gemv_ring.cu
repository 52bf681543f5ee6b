// gemv_ring.cu -- batch-1 decode GEMV fed by a bulk-copy (TMA engine) weight
// ring.
//
// The register-streaming GEMV (gemv.cu) keeps at most one batch of 16-byte
// loads per lane in flight, so each warp walks its rows as a chain of DRAM
// round trips, and its grid needs two CTAs per SM that fill the register
// file: the next kernel of the step cannot become resident until the last
// CTAs leave, and a projection of 30-50 MB is over before the stream reaches
// full rate.  This kernel instead:
//   * gives each SM one CTA of 8 consumer warps plus one producer warp whose
//     elected lane issues cp.async.bulk copies of weight-row chunks into a
//     5-stage x 16 KB shared-memory ring (80 KB in flight per SM, no register
//     cost), tagged L2 evict-first (weights are read once per step);
//   * uses half an SM's registers and about 90 KB of shared memory, so the
//     next kernel's CTA (this kernel again, or the attention) is resident
//     beside it and, with programmatic dependent launch, its producer streams
//     the next projection's weights while this one drains -- the weight
//     stream does not stop at the kernel boundary;
//   * cuts the flattened (task group, K chunk) space into equal contiguous
//     ranges per CTA (stream-K), so every SM streams the same bytes whatever
//     the row count.  A task group (8 consecutive tasks, one per consumer
//     warp) cut between two CTAs leaves fp32 partial dot products in a small
//     scratch; the CTA that completes the group last (arrival counter) sums
//     the parts in CTA order and runs the epilogue.
// A stage holds one K chunk of the group's 8*R rows (R = 2 for the RoPE /
// SwiGLU row pairs): KC = 1024/R halves per row.  Prologues (RMSNorm of the
// fp32 residual stream, or plain half x) and epilogues are those of gemv.cu.
// Used for batch 1 on one GPU (the tensor-parallel exchange keeps the
// register form).
#include "gemv_parts.cuh"
#include "tc.cuh"

namespace b2 {

int* wait_error_word();

constexpr int kRingWarps = 8;                         // consumer warps
constexpr int kRingThreads = 32 * (kRingWarps + 1);   // + the producer warp
constexpr int kRingStageBytes = 16384;
constexpr int kRingStages = 5;

struct RingPlan {
    int C;   // K chunks per task
    int KC;  // halves per chunk row
    int U;   // units = task groups * C
};

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
            "r"(tc::smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(tc::smem_u32(bar)), "l"(pol)
        : "memory");
}

// CTA whose unit range [c*U/grid, (c+1)*U/grid) holds unit u.
__device__ __forceinline__ int ring_cta_of(int u, int U, int grid) {
    return (int)((((int64_t)u + 1) * grid + U - 1) / U) - 1;
}
__device__ __forceinline__ int ring_u0(int c, int U, int grid) { return (int)((int64_t)c * U / grid); }

// Bounded wait that ignores the grid's error word (final drain of copies in
// flight): gives up after about 0.1 s.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
    const long long t0 = clock64();
    while (!tc::mbar_try_wait(bar, parity))
        if (clock64() - t0 > 200000000ll) return;
}

template <int R, int XM, int OM>
__global__ void __launch_bounds__(kRingThreads, 2) gemv_ring_kernel(const GemvParams p, const RingPlan pl) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* ring = smem;                                                        // [stages][16 KB]
    uint4* xs = reinterpret_cast<uint4*>(smem + kRingStages * kRingStageBytes);  // [K8] packed half
    __shared__ __align__(8) uint64_t full[kRingStages], empty[kRingStages];
    __shared__ float s_rs[1];
    __shared__ float s_ss[1][kRingWarps];
    __shared__ unsigned long long s_best[kRingWarps];
    __shared__ int s_last;

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int K = p.K, T = p.tasks, C = pl.C, KC = pl.KC, U = pl.U;
    const int grid = gridDim.x, c = blockIdx.x;
    const int u0 = ring_u0(c, U, grid), u1 = ring_u0(c + 1, U, grid);
    int* err = p.ring_err;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kRingStages; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], kRingWarps);
        }
        tc::fence_barrier_init();
    }
    __syncthreads();
    griddep_launch_dependents();

    if (warp == kRingWarps) {
        // ---- producer: weights do not depend on earlier kernels ----------
        if (lane == 0) {
            uint64_t pol;
            asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
            int it = 0;
            for (int u = u0; u < u1; ++u, ++it) {
                const int slot = it % kRingStages;
                if (it >= kRingStages && !tc::mbar_wait(&empty[slot], ((it / kRingStages) - 1) & 1, err, 301))
                    break;
                const int g = u / C, ch = u - g * C;
                const int k0 = ch * KC, n = min(KC, K - k0);
                const int tasks_here = min(kRingWarps, T - kRingWarps * g);
                tc::mbar_arrive_expect_tx(&full[slot], (uint32_t)(tasks_here * R * n * 2));
                uint8_t* dst = ring + slot * kRingStageBytes;
                for (int w = 0; w < tasks_here; ++w) {
                    const uint4* rp[R];
                    task_rows<R, OM>(p, kRingWarps * g + w, rp);
#pragma unroll
                    for (int r = 0; r < R; ++r)
                        bulk_g2s(dst + (size_t)(w * R + r) * KC * 2, rp[r] + (k0 >> 3), (uint32_t)n * 2, &full[slot],
                                 pol);
                }
            }
            // every copy this CTA issued has landed before it exits
            for (int s = 0; s < kRingStages && s < it; ++s) {
                const int last = s + ((it - 1 - s) / kRingStages) * kRingStages;  // last iteration on slot s
                mbar_drain(&full[s], (last / kRingStages) & 1);
            }
        }
        __syncwarp();
    } else {
        // ---- consumers ---------------------------------------------------
        griddep_wait();
        trace_begin(p.trace);
        stage_x<1, XM, 32 * kRingWarps, 1>(p, xs, s_rs, s_ss, lane, warp);
        unsigned long long best[1] = {0ull};
        const int cg0 = u0 / C;  // the CTA's first group
        int it = 0;
        bool ok = true;
        for (int u = u0; u < u1;) {
            const int g = u / C;
            const int seg_end = min(u1, (g + 1) * C);
            const bool whole = u == g * C && seg_end == (g + 1) * C;
            const int t = kRingWarps * g + warp;
            const bool act = t < T;
            float acc[R][1];
#pragma unroll
            for (int r = 0; r < R; ++r) acc[r][0] = 0.f;
            for (; u < seg_end; ++u, ++it) {
                const int slot = it % kRingStages;
                ok = tc::mbar_wait(&full[slot], (it / kRingStages) & 1, err, 302) && ok;
                if (act && ok) {
                    const int k0 = (u - g * C) * KC;
                    const int n8 = min(KC, K - k0) >> 3;
                    const uint4* wr = reinterpret_cast<const uint4*>(ring + slot * kRingStageBytes) +
                                      (size_t)warp * R * (KC >> 3);
                    const uint4* xr = xs + (k0 >> 3);
#pragma unroll 4
                    for (int q = lane; q < n8; q += 32) {
                        const uint4 xv = xr[q];
#pragma unroll
                        for (int r = 0; r < R; ++r) acc[r][0] = dot8(wr[r * (KC >> 3) + q], xv, acc[r][0]);
                    }
                }
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&empty[slot]);
            }
#pragma unroll
            for (int r = 0; r < R; ++r) acc[r][0] = warp_sum(acc[r][0]);
            if (whole) {
                if (act) task_epilogue<R, 1, OM>(p, t, acc, lane, best, nullptr, 0);
                continue;
            }
            // group cut between CTAs: leave this CTA's part, the last to arrive finishes
            const int which = g == cg0 ? 0 : 1;
            if (lane == 0) {
                float* dst = p.ring_part + (((size_t)c * 2 + which) * kRingWarps + warp) * R;
#pragma unroll
                for (int r = 0; r < R; ++r) __stcg(dst + r, acc[r][0]);
            }
            __threadfence();
            __syncwarp();
            cta_sync<1, 32 * kRingWarps>();
            const int first = ring_cta_of(g * C, U, grid), last = ring_cta_of((g + 1) * C - 1, U, grid);
            if (threadIdx.x == 0) {
                const int old = atomicAdd(p.ring_cnt + g, 1);
                s_last = old == last - first;
                if (s_last) p.ring_cnt[g] = 0;  // ready for the next launch
                __threadfence();
            }
            __syncwarp();
            cta_sync<1, 32 * kRingWarps>();
            if (s_last) {
                float tot[R][1];
#pragma unroll
                for (int r = 0; r < R; ++r) tot[r][0] = 0.f;
                for (int cc = first; cc <= last; ++cc) {
                    const int wh = g == ring_u0(cc, U, grid) / C ? 0 : 1;
                    const float* src = p.ring_part + (((size_t)cc * 2 + wh) * kRingWarps + warp) * R;
#pragma unroll
                    for (int r = 0; r < R; ++r) tot[r][0] += __ldcg(src + r);
                }
                if (act) task_epilogue<R, 1, OM>(p, t, tot, lane, best, nullptr, 0);
            }
        }
        if constexpr (OM == OUT_LOGITS) {
            if (lane == 0) s_best[warp] = best[0];
            __syncwarp();
            cta_sync<1, 32 * kRingWarps>();
            if (threadIdx.x == 0) {
                unsigned long long m = 0ull;
                for (int w = 0; w < kRingWarps; ++w) m = s_best[w] > m ? s_best[w] : m;
                if (m) atomicMax(p.argmax, m);
            }
        }
    }
    __syncthreads();
    trace_end(p.trace);
}

// ---------------------------------------------------------------------------
// launch
// ---------------------------------------------------------------------------
static bool ring_enabled() {
    static int on = -1;
    if (on < 0) {
        const char* e = getenv("B2_GEMV_RING");
        on = (e && e[0] == '0') ? 0 : 1;
    }
    return on == 1;
}

size_t ring_part_floats() { return (size_t)sm_count() * 2 * kRingWarps * 2; }
int ring_groups(int tasks) { return (tasks + kRingWarps - 1) / kRingWarps; }

template <int R, int XM, int OM>
static int launch_ring(const GemvParams& p, cudaStream_t s, bool pdl) {
    auto kern = gemv_ring_kernel<R, XM, OM>;
    const size_t smem = (size_t)kRingStages * kRingStageBytes + (size_t)p.K * sizeof(__half);
    static thread_local int last_dev = -1;
    static thread_local size_t last_smem = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev != last_dev || smem > last_smem) {
        B2_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        last_dev = dev;
        last_smem = smem;
    }
    RingPlan pl;
    pl.KC = 1024 / R;
    pl.C = (p.K + pl.KC - 1) / pl.KC;
    const int G = ring_groups(p.tasks);
    if (G > p.ring_cnt_cap) return B2_ERR_UNSUPPORTED;
    pl.U = G * pl.C;
    const int grid = pl.U < sm_count() ? pl.U : sm_count();
    B2_TRY(launch(kern, dim3((unsigned)grid), dim3(kRingThreads), smem, s, pdl, p, pl));
    return B2_OK;
}

// B2_ERR_UNSUPPORTED when the ring form does not apply (the caller then runs
// gemv_launch).
int gemv_ring_launch(const GemvParams& p, XMode xm, OutMode om, cudaStream_t s, bool pdl) {
    if (!ring_enabled() || p.B != 1 || p.tp_on || xm == X_SUM || om == OUT_PUSH) return B2_ERR_UNSUPPORTED;
    if (!p.ring_part || !p.ring_cnt || !p.ring_err) return B2_ERR_UNSUPPORTED;
    if (p.tasks <= 0) return B2_OK;
    if (p.K <= 0 || (p.K & 7) || !aligned16(p.W) || !aligned16(p.x) || (p.ldx & 7)) return B2_ERR_UNSUPPORTED;
    if ((size_t)p.K * 2 > 48 * 1024) return B2_ERR_UNSUPPORTED;  // x staging beside the 80 KB ring
    if (om == OUT_SWIGLU && !aligned16(p.W2)) return B2_ERR_UNSUPPORTED;
    if (xm == X_NORM && (!p.norm_w || !aligned16(p.norm_w))) return B2_ERR_UNSUPPORTED;
    switch (om) {
        case OUT_HALF: return xm == X_HALF ? launch_ring<1, X_HALF, OUT_HALF>(p, s, pdl) : B2_ERR_UNSUPPORTED;
        case OUT_F32: return xm == X_HALF ? launch_ring<1, X_HALF, OUT_F32>(p, s, pdl) : B2_ERR_UNSUPPORTED;
        case OUT_RESID: return xm == X_HALF ? launch_ring<1, X_HALF, OUT_RESID>(p, s, pdl) : B2_ERR_UNSUPPORTED;
        case OUT_QKV: return xm == X_NORM ? launch_ring<2, X_NORM, OUT_QKV>(p, s, pdl) : B2_ERR_UNSUPPORTED;
        case OUT_SWIGLU: return xm == X_NORM ? launch_ring<2, X_NORM, OUT_SWIGLU>(p, s, pdl) : B2_ERR_UNSUPPORTED;
        case OUT_LOGITS: return xm == X_NORM ? launch_ring<1, X_NORM, OUT_LOGITS>(p, s, pdl) : B2_ERR_UNSUPPORTED;
        default: return B2_ERR_UNSUPPORTED;
    }
}

}  // namespace b2
