// gemv.cu -- decode GEMV family for sm_100a.
//
// Decode at small batch is a pure weight stream: every weight byte is read
// once per step and each is used for B multiply-adds, so the kernel's job is
// to keep enough 16-byte loads in flight to saturate HBM3e and to hide the
// kernel boundary.  Design:
//   * one warp per task (a row, or a pair of rows that its epilogue needs
//     together: the two rotate-half partners of a q/k head, or the gate and up
//     rows of one FFN unit), full K per warp, so no cross-warp reduction;
//   * 128-bit L1-bypassing loads (ld.global.nc.L1::no_allocate.v4), U chunks of
//     16 bytes per lane per row per batch, software pipelined: the next batch
//     of loads is issued before the current one is multiplied, so every lane
//     keeps 2*R*U*16 bytes in flight;
//   * the activation vector is staged once per CTA in shared memory (for the
//     X_NORM forms the RMSNorm of the fp32 residual stream is computed there,
//     fusing the norm kernel away);
//   * grid sized from the SM count and measured occupancy so that every warp
//     gets the same number of tasks (no half-empty last wave);
//   * programmatic dependent launch: the first batch of weight loads is issued
//     before griddepcontrol.wait, overlapping the previous kernel's tail.
// Reference kernel replaced: src/cuda/gemv.cu:28-116 (one warp per row,
// scalar 2-byte loads, separate norm / RoPE / SwiGLU / residual kernels).
#include <cuda_fp8.h>

#include <cmath>
#include <mutex>

#include "gemv_parts.cuh"

namespace b2 {

static int g_sm_count[64];
static std::once_flag g_sm_once[64];

int sm_count() {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    std::call_once(g_sm_once[dev], [dev]() {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        g_sm_count[dev] = n > 0 ? n : 1;
    });
    return g_sm_count[dev];
}

bool pdl_enabled() {
    static int on = -1;
    if (on < 0) {
        const char* e = getenv("B2_PDL");
        on = (e && e[0] == '0') ? 0 : 1;
    }
    return on == 1;
}

// Block size: 256 threads, two CTAs per SM, while the staged activations
// fit twice in shared memory (kGemvSmemPair); else 512 threads and one CTA
// per SM (batch 8 at K = 14336 stages 224 KB), the same 16 warps per SM.
constexpr int kGemvSmemPair = 110 * 1024;
constexpr int kGemvSmemMax = 224 * 1024;

template <int R, int U>
__device__ __forceinline__ void load_rows(uint4 (&w)[R][U], const uint4* const (&rp)[R], int cbase, int K8,
                                          int lane) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int c = cbase + u * 32 + lane;
#pragma unroll
        for (int r = 0; r < R; ++r) w[r][u] = c < K8 ? ldg_stream(rp[r] + c) : make_uint4(0, 0, 0, 0);
    }
}

// Weight formats of the register-streaming GEMV.
enum WFormat { WF_F16 = 0, WF_E4M3 = 1, WF_I4 = 2 };

// Weight row r of matrix m (0: W, 1: W2) as 16-byte chunks: 8 halves, 16
// e4m3 codes, or 32 4-bit codes.
template <int WF>
__device__ __forceinline__ const uint4* weight_row(const GemvParams& p, int m, int r) {
    if constexpr (WF == WF_E4M3)
        return reinterpret_cast<const uint4*>((m ? p.W8b : p.W8) + (size_t)r * p.K);
    else if constexpr (WF == WF_I4)
        return reinterpret_cast<const uint4*>((m ? p.W8b : p.W8) + (size_t)r * (p.K >> 1));
    else
        return reinterpret_cast<const uint4*>((m ? p.W2 : p.W) + (size_t)r * p.K);
}

// Row index and matrix of task t's rows, in the order task_rows gives them.
template <int R, int OM>
__device__ __forceinline__ void task_row_ids(const GemvParams& p, int t, int (&row)[R], int (&mat)[R]) {
    if constexpr (OM == OUT_QKV) {
        const int half = p.D >> 1;
        const int h = t / half, i = t - h * half;
        row[0] = h * p.D + i;
        row[1] = h * p.D + i + half;
        mat[0] = mat[1] = 0;
    } else if constexpr (OM == OUT_SWIGLU) {
        row[0] = row[1] = t;
        mat[0] = 0;
        mat[1] = 1;
    } else {
        row[0] = t;
        mat[0] = 0;
    }
}

template <int R, int OM, int WF>
__device__ __forceinline__ void task_rows(const GemvParams& p, int t, const uint4* (&rp)[R]) {
    int row[R], mat[R];
    task_row_ids<R, OM>(p, t, row, mat);
#pragma unroll
    for (int r = 0; r < R; ++r) rp[r] = weight_row<WF>(p, mat[r], row[r]);
}

// 4-bit weights: the group-scale rows of task t's rows.
template <int R, int OM>
__device__ __forceinline__ void task_group_scales(const GemvParams& p, int t, const float* (&sp)[R]) {
    int row[R], mat[R];
    task_row_ids<R, OM>(p, t, row, mat);
    const int groups = p.K / kI4Group;
#pragma unroll
    for (int r = 0; r < R; ++r) sp[r] = (mat[r] ? p.wsc2 : p.wsc) + (size_t)row[r] * groups;
}

// The scales of the chunks load_rows brings (chunk c of a row lies in group
// c / 4: 32 weights per chunk, 128 per group).
template <int R, int U>
__device__ __forceinline__ void load_group_scales(float (&sc)[R][U], const float* const (&sp)[R], int cbase,
                                                  int KC, int lane) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int c = cbase + u * 32 + lane;
#pragma unroll
        for (int r = 0; r < R; ++r) sc[r][u] = c < KC ? __ldg(sp[r] + (c >> 2)) : 0.f;
    }
}

// One 32-bit word of 4-bit codes (8 weights, kI4Group's bit layout) -> 8
// halves in weight order.  (0x6400 | u) is the half 1024 + u exactly for
// u < 1024, so subtracting 1032 gives u - 8 = q exactly.
__device__ __forceinline__ uint4 i4word_to_half8(uint32_t w) {
    const __half2 bias = __halves2half2(__ushort_as_half((unsigned short)0x6408u),
                                        __ushort_as_half((unsigned short)0x6408u));
    uint32_t o[4];
#pragma unroll
    for (int pr = 0; pr < 4; ++pr) {
        const uint32_t v = ((w >> (4 * pr)) & 0x000F000Fu) | 0x64006400u;
        const __half2 h = __hsub2(*reinterpret_cast<const __half2*>(&v), bias);
        o[pr] = *reinterpret_cast<const uint32_t*>(&h);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// Per-row scales of task t's rows (FP8 weights), in task_rows' order.
template <int R, int OM>
__device__ __forceinline__ void task_scales(const GemvParams& p, int t, float (&sc)[R]) {
    if constexpr (OM == OUT_QKV) {
        const int half = p.D >> 1;
        const int h = t / half, i = t - h * half;
        sc[0] = p.wsc[h * p.D + i];
        sc[1] = p.wsc[h * p.D + i + half];
    } else if constexpr (OM == OUT_SWIGLU) {
        sc[0] = p.wsc[t];
        sc[1] = p.wsc2[t];
    } else {
        sc[0] = p.wsc[t];
    }
}

// 16 e4m3 codes -> two chunks of 8 halves (exact: every e4m3 value is a
// half), in element order.
__device__ __forceinline__ void e4m3x16_to_half(const uint4& w, uint4& lo, uint4& hi) {
    auto cvt2 = [](uint32_t bits16) -> uint32_t {
        const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)bits16, __NV_E4M3);
        return (uint32_t)h.x | ((uint32_t)h.y << 16);
    };
    lo.x = cvt2(w.x & 0xffffu);
    lo.y = cvt2(w.x >> 16);
    lo.z = cvt2(w.y & 0xffffu);
    lo.w = cvt2(w.y >> 16);
    hi.x = cvt2(w.z & 0xffffu);
    hi.y = cvt2(w.z >> 16);
    hi.z = cvt2(w.w & 0xffffu);
    hi.w = cvt2(w.w >> 16);
}


// ---------------------------------------------------------------------------
// register-streaming form
// ---------------------------------------------------------------------------
// CTAs per SM the register budget is sized for.  Three 256-thread CTAs (80
// registers) for the batch-1 q|k|v and lm_head GEMVs: their tasks then go out
// in one round instead of two (Llama-3-8B q|k|v: 12.2 -> 9.8 us); the o and
// down GEMVs lose more to the tighter register budget than they gain (down
// 19.7 -> 23.0 us), and the exchange consumers would spill.
// (4-bit weights keep two: their dequantisation needs the registers, and
// with 80 the q|k|v and lm_head forms spill.)
constexpr int gemv_min_ctas(int NT, int BT, int XM, int OM, int WF) {
    return NT != 256 ? 1 : (BT == 1 && XM != X_SUM && (OM == OUT_QKV || OM == OUT_LOGITS) && WF != WF_I4) ? 3 : 2;
}

template <int R, int BT, int XM, int OM, int U, int WF, int NT>
__global__ void __launch_bounds__(NT, gemv_min_ctas(NT, BT, XM, OM, WF)) gemv_vec_kernel(const GemvParams p) {
    constexpr int kGemvWarps = NT / 32;
    extern __shared__ __align__(16) uint4 xs[];  // [BT][K8] packed half
    __shared__ float s_rs[BT];
    __shared__ float s_ss[BT][kGemvWarps];
    __shared__ unsigned long long s_best[kGemvWarps][BT];
    __shared__ __align__(16) float s_push[OM == OUT_PUSH ? BT * kPushRows : 1];

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int K8 = p.K >> 3;                  // 16-byte chunks of x (8 halves)
    const int KC = WF == WF_E4M3 ? (p.K >> 4) : WF == WF_I4 ? (p.K >> 5) : K8;  // 16-byte chunks of a weight row
    const int NB = (KC + 32 * U - 1) / (32 * U);
    // Tasks are dealt round-robin over all warps of the grid, except for
    // OUT_PUSH, where each CTA owns a contiguous block of rows so that it can
    // push them to the other ranks as 16-byte stores once its stream is done.
    constexpr bool kBlockRows = OM == OUT_PUSH;
    const int total_warps = gridDim.x * kGemvWarps;
    const int row0 = kBlockRows ? blockIdx.x * p.rows_per_cta : 0;
    const int t_step = kBlockRows ? kGemvWarps : total_warps;
    const int t_end = kBlockRows ? min(p.tasks, row0 + p.rows_per_cta) : p.tasks;
    int t = kBlockRows ? row0 + warp : blockIdx.x * kGemvWarps + warp;

    // Weights do not depend on the previous kernel: start streaming them now.
    uint4 wn[R][U];
    float sn[R][U];  // 4-bit weights: the chunks' group scales
    if (t < t_end) {
        const uint4* rp[R];
        task_rows<R, OM, WF>(p, t, rp);
        load_rows<R, U>(wn, rp, 0, KC, lane);
        if constexpr (WF == WF_I4) {
            const float* sp[R];
            task_group_scales<R, OM>(p, t, sp);
            load_group_scales<R, U>(sn, sp, 0, KC, lane);
        }
    }

    // X_SUM reads the previous kernel's output only through the tagged
    // exchange words it polls, and everything else it reads or overwrites was
    // last touched two or more kernels back (whose completion the previous
    // kernel's own wait implied), so it skips the programmatic-launch wait
    // and starts polling as soon as it is resident.
    if constexpr (XM != X_SUM) griddep_wait();
    griddep_launch_dependents();
    trace_begin(p.trace);

    stage_x<BT, XM, NT>(p, xs, s_rs, s_ss, lane, warp);

    unsigned long long best[BT];
#pragma unroll
    for (int b = 0; b < BT; ++b) best[b] = 0ull;
    unsigned push_epoch = 0, push_par = 0;
    if constexpr (OM == OUT_PUSH) {
        push_epoch = (unsigned)(*p.tpx.step) * (unsigned)p.nslots + (unsigned)p.slot + 1u;
        push_par = push_epoch & 1u;
    }

    // ---- stream the warp's tasks ---------------------------------------
    for (; t < t_end; t += t_step) {
        float acc[R][BT];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int b = 0; b < BT; ++b) acc[r][b] = 0.f;

        for (int cb = 0; cb < NB; ++cb) {
            uint4 wc[R][U];
            float scc[R][U];
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    wc[r][u] = wn[r][u];
                    if constexpr (WF == WF_I4) scc[r][u] = sn[r][u];
                }
            // issue the next batch (this task's next chunk batch, or the next task's first)
            {
                int nt = t, ncb = cb + 1;
                if (ncb == NB) { nt = t + t_step; ncb = 0; }
                if (nt < t_end) {
                    const uint4* rp[R];
                    task_rows<R, OM, WF>(p, nt, rp);
                    load_rows<R, U>(wn, rp, ncb * 32 * U, KC, lane);
                    if constexpr (WF == WF_I4) {
                        const float* sp[R];
                        task_group_scales<R, OM>(p, nt, sp);
                        load_group_scales<R, U>(sn, sp, ncb * 32 * U, KC, lane);
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = cb * 32 * U + u * 32 + lane;
                if (c < KC) {
                    if constexpr (WF == WF_I4) {  // 32 weights: x chunks 4c .. 4c + 3, one group scale
                        uint4 hw[R][4];
#pragma unroll
                        for (int r = 0; r < R; ++r) {
                            hw[r][0] = i4word_to_half8(wc[r][u].x);
                            hw[r][1] = i4word_to_half8(wc[r][u].y);
                            hw[r][2] = i4word_to_half8(wc[r][u].z);
                            hw[r][3] = i4word_to_half8(wc[r][u].w);
                        }
#pragma unroll
                        for (int b = 0; b < BT; ++b) {
                            const uint4* xb = xs + b * K8 + 4 * c;
                            const uint4 x0 = xb[0], x1 = xb[1], x2 = xb[2], x3 = xb[3];
#pragma unroll
                            for (int r = 0; r < R; ++r) {
                                float part = dot8_mixed(hw[r][0], x0, 0.f);
                                part = dot8_mixed(hw[r][1], x1, part);
                                part = dot8_mixed(hw[r][2], x2, part);
                                part = dot8_mixed(hw[r][3], x3, part);
                                acc[r][b] = fmaf(part, scc[r][u], acc[r][b]);
                            }
                        }
                    } else if constexpr (WF == WF_E4M3) {  // 16 weights: x chunks 2c and 2c + 1
                        uint4 lo[R], hi[R];
#pragma unroll
                        for (int r = 0; r < R; ++r) e4m3x16_to_half(wc[r][u], lo[r], hi[r]);
#pragma unroll
                        for (int b = 0; b < BT; ++b) {
                            const uint4 x0 = xs[b * K8 + 2 * c], x1 = xs[b * K8 + 2 * c + 1];
#pragma unroll
                            for (int r = 0; r < R; ++r) acc[r][b] = dot8_mixed(hi[r], x1, dot8_mixed(lo[r], x0, acc[r][b]));
                        }
                    } else {
#pragma unroll
                        for (int b = 0; b < BT; ++b) {
                            const uint4 xv = xs[b * K8 + c];
#pragma unroll
                            for (int r = 0; r < R; ++r) acc[r][b] = dot8_mixed(wc[r][u], xv, acc[r][b]);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int b = 0; b < BT; ++b) acc[r][b] = warp_sum(acc[r][b]);
        if constexpr (WF == WF_E4M3) {  // the rows' scales
            float sc[R];
            task_scales<R, OM>(p, t, sc);
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int b = 0; b < BT; ++b) acc[r][b] *= sc[r];
        }
        task_epilogue<R, BT, OM>(p, t, acc, lane, best, s_push, row0);
    }

    gemv_finish<BT, OM, NT>(p, lane, warp, best, s_best, s_push, row0, t_end, push_epoch, push_par);
    __syncthreads();
    trace_end(p.trace);
    // X_SUM: no CTA leaves while a cluster peer may still read its slice of h
    if constexpr (XM == X_SUM) cluster_wait_acquire();
}

// ---------------------------------------------------------------------------
// launch plumbing
// ---------------------------------------------------------------------------

// Thread-block cluster size of the X_SUM (exchange-consumer) GEMVs: the CTAs
// of a cluster share the reads of the exchange words (B2_XSUM_CLUSTER
// overrides, 1..8).
static int xsum_cluster() {
    static int cs = -1;
    if (cs < 0) {
        const char* e = getenv("B2_XSUM_CLUSTER");
        const int v = e ? atoi(e) : 8;
        cs = v >= 1 && v <= 8 ? v : 8;
    }
    return cs;
}

// Dynamic shared memory of a launch: x staged as halves, and (X_SUM) this
// CTA's slice of the fp32 residual.
static size_t gemv_smem(int BT, int XM, int K, int cs) {
    return (size_t)BT * K * sizeof(__half) +
           (XM == X_SUM ? (size_t)BT * (((K >> 3) + cs - 1) / cs) * 8 * sizeof(float) : 0);
}

template <int R, int BT, int XM, int OM, int U, int WF, int NT>
static int launch_vec(const GemvParams& p, cudaStream_t s, bool pdl) {
    constexpr int kGemvThreads = NT, kGemvWarps = NT / 32;
    auto kern = gemv_vec_kernel<R, BT, XM, OM, U, WF, NT>;
    const int cs = XM == X_SUM ? xsum_cluster() : 1;
    const size_t smem = gemv_smem(BT, XM, p.K, cs);
    if (smem > (size_t)kGemvSmemMax) return B2_ERR_UNSUPPORTED;
    // per-device occupancy cache, keyed on the shared-memory footprint
    static thread_local int last_dev = -1;
    static thread_local size_t last_smem = (size_t)-1;
    static thread_local int last_occ = 1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev != last_dev || smem != last_smem) {
        B2_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(smem > 0 ? smem : 1)));
        int occ = 0;
        if (XM == X_SUM) {
            // co-resident CTAs in whole clusters (a cluster sits in one GPC)
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3((unsigned)(cs * sm_count()));
            cfg.blockDim = dim3(kGemvThreads);
            cfg.dynamicSmemBytes = smem;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = (unsigned)cs;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            int clusters = 0;
            B2_TRY(cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg));
            occ = clusters * cs;  // CTAs device-wide
        } else {
            B2_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kGemvThreads, smem));
            occ *= sm_count();
        }
        last_occ = occ > 0 ? occ : cs;
        last_dev = dev;
        last_smem = smem;
    }
    const int max_warps = last_occ * kGemvWarps;
    const int rounds = (p.tasks + max_warps - 1) / max_warps;
    const int warps = (p.tasks + rounds - 1) / rounds;
    int ctas = (warps + kGemvWarps - 1) / kGemvWarps;
    if (cs > 1) ctas = (ctas + cs - 1) / cs * cs;
    GemvParams q = p;
    if (OM == OUT_PUSH) {
        q.rows_per_cta = kGemvWarps * rounds;
        if (q.rows_per_cta > kPushRows || (p.tasks & 7)) return B2_ERR_UNSUPPORTED;
        ctas = (p.tasks + q.rows_per_cta - 1) / q.rows_per_cta;
    }
    if (XM == X_SUM)
        B2_TRY(launch_cluster(kern, dim3(ctas), dim3(kGemvThreads), smem, s, pdl, (unsigned)cs, q));
    else
        B2_TRY(launch(kern, dim3(ctas), dim3(kGemvThreads), smem, s, pdl, q));
    return B2_OK;
}

int gemv_batch_tile(int K) {
    // x staging of one CTA (one per SM past kGemvSmemPair) within kGemvSmemMax
    for (int bt = 8; bt > 1; bt >>= 1)
        if ((long)bt * K * 2 <= kGemvSmemMax) return bt;
    return 1;
}

template <int R, int BT, int XM, int OM, int U, int WF>
static int launch_nt(const GemvParams& p, cudaStream_t s, bool pdl) {
    const int cs = XM == X_SUM ? xsum_cluster() : 1;
    if (gemv_smem(BT, XM, p.K, cs) <= (size_t)kGemvSmemPair) return launch_vec<R, BT, XM, OM, U, WF, 256>(p, s, pdl);
    return launch_vec<R, BT, XM, OM, U, WF, 512>(p, s, pdl);
}

template <int R, int XM, int OM, int U, int WF>
static int dispatch_bt_w(const GemvParams& p, cudaStream_t s, bool pdl) {
    if (p.B <= 1) return launch_nt<R, 1, XM, OM, U, WF>(p, s, pdl);
    if (p.B <= 2) return launch_nt<R, 2, XM, OM, U, WF>(p, s, pdl);
    if constexpr (WF == WF_I4) {
        return B2_ERR_UNSUPPORTED;  // 4-bit weights: batch tiles of 1 and 2
    } else {
        if (p.B <= 4) return launch_nt<R, 4, XM, OM, U, WF>(p, s, pdl);
        return launch_nt<R, 8, XM, OM, U, WF>(p, s, pdl);
    }
}

// FP8 weights: 16-byte chunks of 16 codes, 4-bit weights: of 32 codes (U
// chunks per lane and batch, as for halves, so the same bytes are in flight
// with two or four times the weights).
template <int R, int XM, int OM, int U>
static int dispatch_bt(const GemvParams& p, cudaStream_t s, bool pdl) {
    if (p.W8 && p.w4) return dispatch_bt_w<R, XM, OM, U, WF_I4>(p, s, pdl);
    if (p.W8) return dispatch_bt_w<R, XM, OM, U, WF_E4M3>(p, s, pdl);
    return dispatch_bt_w<R, XM, OM, U, WF_F16>(p, s, pdl);
}

int gemv_launch(const GemvParams& p, XMode xm, OutMode om, cudaStream_t s, bool pdl) {
    if (p.tasks <= 0 || p.B <= 0) return B2_OK;
    if (p.K <= 0 || (p.K & 7) || !aligned16(p.x) || (p.ldx & 7)) return B2_ERR_UNSUPPORTED;
    if (p.W8 ? ((p.K & (p.w4 ? kI4Group - 1 : 15)) || !aligned16(p.W8) || !p.wsc ||
                (om == OUT_SWIGLU && (!aligned16(p.W8b) || !p.wsc2)))
             : !aligned16(p.W))
        return B2_ERR_UNSUPPORTED;
    if (p.W8 && p.w4 && p.B > 2) return B2_ERR_UNSUPPORTED;
    if (p.B > 8 || p.B > gemv_batch_tile(p.K)) return B2_ERR_UNSUPPORTED;
    if (om == OUT_SWIGLU && !p.W8 && !aligned16(p.W2)) return B2_ERR_UNSUPPORTED;
    if ((xm == X_NORM || xm == X_SUM) && (!p.norm_w || !aligned16(p.norm_w))) return B2_ERR_UNSUPPORTED;
    if ((xm == X_SUM || om == OUT_PUSH) && (!p.tp_on || p.tpx.tp < 1 || p.tpx.tp > kMaxTp)) return B2_ERR_INVALID;
    switch (om) {
        case OUT_HALF: return dispatch_bt<1, X_HALF, OUT_HALF, 8>(p, s, pdl);
        case OUT_F32:  return dispatch_bt<1, X_HALF, OUT_F32, 8>(p, s, pdl);
        case OUT_RESID: return dispatch_bt<1, X_HALF, OUT_RESID, 8>(p, s, pdl);
        case OUT_PUSH: return p.tp_on ? dispatch_bt<1, X_HALF, OUT_PUSH, 8>(p, s, pdl) : B2_ERR_INVALID;
        case OUT_QKV:
            if (xm == X_SUM) return dispatch_bt<2, X_SUM, OUT_QKV, 4>(p, s, pdl);
            return xm == X_NORM ? dispatch_bt<2, X_NORM, OUT_QKV, 4>(p, s, pdl) : B2_ERR_UNSUPPORTED;
        case OUT_SWIGLU:
            if (xm == X_SUM) return dispatch_bt<2, X_SUM, OUT_SWIGLU, 4>(p, s, pdl);
            return xm == X_NORM ? dispatch_bt<2, X_NORM, OUT_SWIGLU, 4>(p, s, pdl) : B2_ERR_UNSUPPORTED;
        case OUT_LOGITS:
            if (xm == X_SUM) return dispatch_bt<1, X_SUM, OUT_LOGITS, 8>(p, s, pdl);
            return xm == X_NORM ? dispatch_bt<1, X_NORM, OUT_LOGITS, 8>(p, s, pdl) : B2_ERR_UNSUPPORTED;
    }
    return B2_ERR_UNSUPPORTED;
}

// ---------------------------------------------------------------------------
// generic path: any K, any alignment (odd API shapes).  One warp per row.
// ---------------------------------------------------------------------------
__global__ void gemv_generic_kernel(const __half* __restrict__ W, const __half* __restrict__ x,
                                    const __half* __restrict__ extra, void* __restrict__ y, int B, int N,
                                    int K, int epi, int out_f32) {
    griddep_wait();
    const int lane = threadIdx.x & 31;
    const int nw = (gridDim.x * blockDim.x) >> 5;
    for (int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < N; row += nw) {
        const __half* wr = W + (size_t)row * K;
        for (int b = 0; b < B; ++b) {
            const __half* xb = x + (size_t)b * K;
            float acc = 0.f;
            for (int k = lane; k < K; k += 32) acc = fmaf(__half2float(wr[k]), __half2float(xb[k]), acc);
            acc = warp_sum(acc);
            if (lane == 0) {
                if (epi == 1) acc += __half2float(extra[row]);
                if (epi == 2) acc += __half2float(extra[(size_t)b * N + row]);
                if (out_f32) static_cast<float*>(y)[(size_t)b * N + row] = acc;
                else static_cast<__half*>(y)[(size_t)b * N + row] = __float2half_rn(acc);
            }
        }
    }
}

static int gemv_api(const void* W, const void* x, const void* extra, void* y, int B, int N, int K, int epi,
                    int out_f32, void* stream) {
    if (N <= 0 || K <= 0 || B <= 0) return B2_OK;
    B2_REQUIRE(W && x && y && (epi == 0 || extra));
    B2_REQUIRE(epi >= 0 && epi <= 2);
    cudaStream_t s = as_stream(stream);
    const bool vec_ok = (K % 8 == 0) && aligned16(W) && aligned16(x);
    if (vec_ok) {
        const int bt = gemv_batch_tile(K);
        for (int b0 = 0; b0 < B; b0 += bt) {
            const int nb = B - b0 < bt ? B - b0 : bt;
            GemvParams p = {};
            p.W = static_cast<const __half*>(W);
            p.K = K;
            p.tasks = N;
            p.B = nb;
            p.x = static_cast<const __half*>(x) + (size_t)b0 * K;
            p.ldx = K;
            p.bias = epi == 1 ? static_cast<const __half*>(extra) : nullptr;
            p.resid = epi == 2 ? static_cast<const __half*>(extra) + (size_t)b0 * N : nullptr;
            p.ld_resid = N;
            p.y = out_f32 ? (void*)(static_cast<float*>(y) + (size_t)b0 * N)
                          : (void*)(static_cast<__half*>(y) + (size_t)b0 * N);
            p.ldy = N;
            const int rc = gemv_launch(p, X_HALF, out_f32 ? OUT_F32 : OUT_HALF, s, true);
            if (rc != B2_OK) return rc;
        }
        return B2_OK;
    }
    const int threads = 256;
    long ctas = ((long)N * 32 + threads - 1) / threads;
    const long cap = (long)sm_count() * 8;
    if (ctas > cap) ctas = cap;
    B2_TRY(launch(gemv_generic_kernel, dim3((unsigned)ctas), dim3(threads), 0, s, true,
                  static_cast<const __half*>(W), static_cast<const __half*>(x), static_cast<const __half*>(extra), y,
                  B, N, K, epi, out_f32));
    return B2_OK;
}

}  // namespace b2

extern "C" int b2_gemv(const void* W, const void* x, void* y, int N, int K, void* stream) {
    return b2::gemv_api(W, x, nullptr, y, 1, N, K, 0, 0, stream);
}

extern "C" int b2_gemv_bias(const void* W, const void* x, const void* b, void* y, int N, int K, void* stream) {
    return b2::gemv_api(W, x, b, y, 1, N, K, 1, 0, stream);
}

extern "C" int b2_gemv_residual(const void* W, const void* x, const void* r, void* y, int N, int K, void* stream) {
    return b2::gemv_api(W, x, r, y, 1, N, K, 2, 0, stream);
}

extern "C" int b2_gemv_batched(const void* W, const void* x, const void* extra, void* y, int B, int N, int K,
                               int epilogue, int out_f32, void* stream) {
    return b2::gemv_api(W, x, extra, y, B, N, K, epilogue, out_f32, stream);
}
