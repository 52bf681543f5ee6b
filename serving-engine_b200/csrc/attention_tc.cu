// attention_tc.cu -- split-KV GQA decode attention on the tcgen05 tensor
// cores (head_dim 128), sm_100a.
//
// Decode attention is a K/V stream: per (sequence, kv head) the group's query
// heads (<= 8) meet every cached position once.  Both products run on the
// tensor cores with the positions on the MMA's M side, so the per-position
// arithmetic that bounds a CUDA-core kernel (dot-product shuffles, 8-wide
// FMAs per head) becomes two MMAs per 128-position tile:
//   S^T = K Q^T     M = 128 positions, N = 16 (the group's heads, zero rows
//                   past them), K = 128 (head dim)     -> TMEM, 2 buffers
//   O^T += V^T P^T  M = 128 (head dim, V read MN-major from the same tile),
//                   N = 16 heads, K = 128 positions    -> TMEM
// Grid and merge as attention_cl.cu: one thread-block cluster of CS <= 8
// CTAs per (sequence, kv head x head group), each CTA a contiguous chunk of
// positions (whole tiles), the CS partials merged through distributed shared
// memory.  Per CTA (192 threads, one CTA per SM):
//   warp 4      TMA producer: K and V tiles (128 positions x 128, 128-byte
//               swizzle, 4-D tensor map over the cache view) into a ring of
//               3 stages (fewer beside register-streaming GEMVs); in the
//               decode step all tiles go out before the programmatic-launch
//               wait and the newest row is copied into its tile after it;
//   warp 5      MMA issuer: S_j, then O += P_{j-1} V_{j-1};
//   warps 0..3  thread t = position t of the tile: its S row (16 heads) from
//               TMEM, scale and mask, per-head tile max across the 128
//               threads, P_j = 2^(S - m) into one of two shared-memory P^T
//               buffers, running sums per thread; O^T columns rescaled in
//               TMEM only when a head's max grows by more than 2^8; at the
//               end thread t holds O^T lane t (= head-dim element t).
// Every mbarrier wait is bounded (tc.cuh).
// Reference replaced: src/cuda/decode_attention_split.cu:28-214 and
// src/cuda/decode_attention.cu:15-141.
#include <cmath>

#include <cooperative_groups.h>

#include "attention.cuh"
#include "tc.cuh"

namespace cg = cooperative_groups;

namespace b2 {

struct AttnTcParams {
    const __half* q;
    int64_t q_sb;
    __half* out;
    int64_t o_sb;
    const int* seq_lens;
    int len_const;
    int nq, nkv, group, hg;
    float scale_log2;
    int early_kv;
    int head_inner;
    const __half* kp;  // the cache views as pointers (the newest row is copied in directly)
    const __half* vp;
    int64_t sb, sh, ss;
    // paged cache (bt != null): block tables [B][maxb] of bs-position blocks,
    // pools [num_blocks][bs][nkv][128]; the tensor maps then cover one block
    const int* bt;
    int maxb, bs;
    int* err;
    TraceSlot trace;
};

constexpr int kAtD = 128;                       // head dim
constexpr int kAtP = 128;                       // positions per tile
constexpr int kAtN = 16;                        // MMA N: heads (padded)
constexpr int kAtMaxCluster = 8;
constexpr uint32_t kAtAtom = 128 * 128;         // 128 rows x 128 bytes
constexpr uint32_t kAtKV = 2 * kAtAtom;         // one K or V tile
constexpr uint32_t kAtStage = 2 * kAtKV;        // K + V
constexpr uint32_t kAtQAtom = kAtN * 128;       // 16 rows x 128 bytes
constexpr uint32_t kAtQBytes = 2 * kAtQAtom;    // Q: 16 heads x 128
constexpr uint32_t kAtPBytes = 2 * kAtQAtom;    // P^T: 16 heads x 128 positions
// shared memory: STAGES K/V stages | Q | 2 P^T buffers | barriers
template <int STAGES>
struct AtSmem {
    static constexpr uint32_t OFF_Q = STAGES * kAtStage;
    static constexpr uint32_t OFF_P = OFF_Q + kAtQBytes;
    static constexpr uint32_t OFF_BAR = OFF_P + 2 * kAtPBytes;
    static constexpr size_t BYTES = OFF_BAR + 256 + 1024;
};
constexpr uint32_t kAtTmemCols = 64;            // S buffers at 0 and 16, O^T at 32
constexpr uint32_t kAtColO = 32;

__device__ __forceinline__ float at_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ void softmax_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// byte offset of element (row, col) in a K-major 128-byte-swizzled operand
// made of 64-column atoms `atom` bytes apart
__device__ __forceinline__ uint32_t at_sw128(int row, int col, uint32_t atom) {
    return (uint32_t)(col >> 6) * atom + (uint32_t)row * 128u + ((((uint32_t)(col & 63) >> 3) ^ (row & 7)) << 4) +
           ((uint32_t)(col & 7) << 1);
}

template <int G, int kAtStages>
__global__ void __launch_bounds__(192, 1) attn_tc_kernel(const __grid_constant__ CUtensorMap tmK,
                                                         const __grid_constant__ CUtensorMap tmV,
                                                         const AttnTcParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* ring = sm;
    using Lay = AtSmem<kAtStages>;
    uint8_t* sQ = sm + Lay::OFF_Q;
    uint8_t* sP = sm + Lay::OFF_P;
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm + Lay::OFF_BAR);
    uint64_t* kv_full = bar + 0;                // [STAGES]
    uint64_t* kv_empty = bar + kAtStages;       // [STAGES]
    uint64_t* q_ready = bar + 2 * kAtStages;
    uint64_t* s_full = q_ready + 1;             // [2]
    uint64_t* p_full = q_ready + 3;             // [2]
    uint64_t* o_done = q_ready + 5;             // [2]: O += P_j V_j done, on o_done[j & 1]
    uint64_t* patch_bar = q_ready + 7;          // newest row copied into its tile
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(q_ready + 8);
    __shared__ float s_red[2][4][G];
    __shared__ float s_lsum[4][G];
    __shared__ float2 s_pm[G];
    __shared__ __align__(16) float s_pa[G][kAtD];
    __shared__ float s_wt[G][kAtMaxCluster];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cs = (int)gridDim.x;
    const int split = blockIdx.x;
    const int kvh = blockIdx.y / p.hg, hgi = blockIdx.y - (blockIdx.y / p.hg) * p.hg;
    const int b = blockIdx.z;
    const int h0 = kvh * p.group + hgi * G;
    const int nh = min(G, p.group - hgi * G);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kAtStages; ++s) {
            tc::mbar_init(&kv_full[s], 1);
            tc::mbar_init(&kv_empty[s], 1);
        }
        tc::mbar_init(q_ready, 128);
        for (int s = 0; s < 2; ++s) {
            tc::mbar_init(&s_full[s], 1);
            tc::mbar_init(&p_full[s], 128);
            tc::mbar_init(&o_done[s], 1);
        }
        tc::mbar_init(patch_bar, 1);
        tc::fence_barrier_init();
    }
    // Q and both P^T buffers start at zero (rows past the group's heads stay zero)
    for (uint32_t i = threadIdx.x; i < (kAtQBytes + 2 * kAtPBytes) / 16; i += blockDim.x)
        reinterpret_cast<uint4*>(sQ)[i] = make_uint4(0, 0, 0, 0);
    tc::fence_proxy_async_smem();
    if (warp == 0) tc::tmem_alloc(tmem_slot, kAtTmemCols);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    if (!p.early_kv) griddep_wait();

    const int L = p.seq_lens ? p.seq_lens[b] : p.len_const;
    int chunk = (L + cs - 1) / cs;
    chunk = ((chunk + kAtP - 1) / kAtP) * kAtP;
    if (chunk < kAtP) chunk = kAtP;
    const int n_used = L > 0 ? (L + chunk - 1) / chunk : 0;
    const bool active = split < n_used;
    const int start = split * chunk;
    const int end = active ? min(L, start + chunk) : start;
    const int nt = active ? (end - start + kAtP - 1) / kAtP : 0;

    float m_run[G], l_th[G];
#pragma unroll
    for (int h = 0; h < G; ++h) {
        m_run[h] = -INFINITY;
        l_th[h] = 0.f;
    }
    uint32_t o_reg[16];
#pragma unroll
    for (int h = 0; h < 16; ++h) o_reg[h] = 0u;

    if (warp == 4) {
        // ---------------- TMA producer ----------------
        // Decode step: every tile goes out before the programmatic-launch
        // wait.  The newest row (position L - 1) is being written by the
        // previous kernel, so whatever its tile brought for it is replaced,
        // after the wait and after that tile has landed, by the row read
        // from the cache directly; the MMA waits for that copy on patch_bar.
        const bool patch = p.early_kv && active && end == L;
        if (lane == 0) {
            for (int i = 0; i < nt; ++i) {
                const int s = i % kAtStages;
                if (i >= kAtStages &&
                    !tc::mbar_wait(&kv_empty[s], (uint32_t)((i / kAtStages) - 1) & 1u, p.err, 71))
                    break;
                const int pos0 = start + i * kAtP;
                uint8_t* st = ring + (size_t)s * kAtStage;
                tc::mbar_arrive_expect_tx(&kv_full[s], kAtStage);
                if (p.bt) {
                    // one box per (block, 64-column atom): rows of block j of
                    // the tile land at row 16j.. of the swizzled tile (a
                    // block is a whole number of 8-row swizzle atoms); table
                    // slots past the sequence's blocks read block 0 (masked)
                    const int nblk = kAtP / p.bs;
                    for (int j = 0; j < nblk; ++j) {
                        const int lb = pos0 / p.bs + j;
                        const int phys = lb < p.maxb ? p.bt[(int64_t)b * p.maxb + lb] : 0;
#pragma unroll
                        for (int a = 0; a < 2; ++a) {
                            const uint32_t off = a * kAtAtom + (uint32_t)(j * p.bs) * 128u;
                            tc::tma_load_4d(st + off, &tmK, &kv_full[s], a * 64, kvh, 0, phys);
                            tc::tma_load_4d(st + kAtKV + off, &tmV, &kv_full[s], a * 64, kvh, 0, phys);
                        }
                    }
                    continue;
                }
#pragma unroll
                for (int a = 0; a < 2; ++a) {
                    if (p.head_inner) {
                        tc::tma_load_4d(st + a * kAtAtom, &tmK, &kv_full[s], a * 64, kvh, pos0, b);
                        tc::tma_load_4d(st + kAtKV + a * kAtAtom, &tmV, &kv_full[s], a * 64, kvh, pos0, b);
                    } else {
                        tc::tma_load_4d(st + a * kAtAtom, &tmK, &kv_full[s], a * 64, pos0, kvh, b);
                        tc::tma_load_4d(st + kAtKV + a * kAtAtom, &tmV, &kv_full[s], a * 64, pos0, kvh, b);
                    }
                }
            }
        }
        __syncwarp();
        griddep_wait();
        if (patch) {
            const int i = nt - 1, s = i % kAtStages;
            const int row = (L - 1) - (start + i * kAtP);
            const bool ok = __all_sync(0xffffffffu, tc::mbar_wait(&kv_full[s], (uint32_t)(i / kAtStages) & 1u, p.err, 79));
            if (ok) {
                const int c = lane & 15;  // 16-byte chunk of the K (lanes 0-15) or V (16-31) row
                const int64_t at = p.bt ? (((int64_t)p.bt[(int64_t)b * p.maxb + (L - 1) / p.bs] * p.bs + (L - 1) % p.bs) *
                                               p.nkv + kvh) * kAtD
                                        : (int64_t)b * p.sb + (int64_t)kvh * p.sh + (int64_t)(L - 1) * p.ss;
                const __half* src = (lane < 16 ? p.kp : p.vp) + at + c * 8;
                uint8_t* dst = ring + (size_t)s * kAtStage + (lane < 16 ? 0u : kAtKV) + (uint32_t)(c >> 3) * kAtAtom +
                               (uint32_t)row * 128u + ((((uint32_t)c & 7u) ^ ((uint32_t)row & 7u)) << 4);
                *reinterpret_cast<uint4*>(dst) = __ldcg(reinterpret_cast<const uint4*>(src));
                tc::fence_proxy_async_smem();
            }
            __syncwarp();
            if (lane == 0 && ok) tc::mbar_arrive(patch_bar);
        }
        griddep_launch_dependents();
    } else if (warp == 5) {
        // ---------------- MMA issuer ----------------
        const bool patch = p.early_kv && active && end == L;
        if (lane == 0 && nt > 0) {
            constexpr uint32_t idS = tc::idesc_f16(128, kAtN, false, false);
            constexpr uint32_t idO = tc::idesc_f16(128, kAtN, false, false, true);
            const uint32_t aQ = tc::smem_u32(sQ), aP = tc::smem_u32(sP), aR = tc::smem_u32(ring);
            bool ok = tc::mbar_wait(q_ready, 0, p.err, 72);
            auto issue_s = [&](int j) -> bool {
                const int s = j % kAtStages;
                bool good = tc::mbar_wait(&kv_full[s], (uint32_t)(j / kAtStages) & 1u, p.err, 73);
                if (good && patch && j == nt - 1) good = tc::mbar_wait(patch_bar, 0, p.err, 80);
                if (!good) return false;
                tc::fence_after_sync();
                const uint32_t aK = aR + (uint32_t)s * kAtStage;
#pragma unroll
                for (int kk = 0; kk < kAtD / 16; ++kk) {
                    const uint32_t offk = (uint32_t)(kk >> 2) * kAtAtom + (uint32_t)(kk & 3) * 32;
                    const uint32_t offq = (uint32_t)(kk >> 2) * kAtQAtom + (uint32_t)(kk & 3) * 32;
                    tc::mma_f16(tmem + (uint32_t)(j & 1) * 16, tc::desc_k_sw128(aK + offk),
                                tc::desc_k_sw128(aQ + offq), idS, kk > 0 ? 1u : 0u);
                }
                tc::mma_commit(&s_full[j & 1]);
                return true;
            };
            auto issue_pv = [&](int jj) -> bool {
                const int sv = jj % kAtStages;
                if (!tc::mbar_wait(&p_full[jj & 1], (uint32_t)(jj >> 1) & 1u, p.err, 74)) return false;
                tc::fence_after_sync();
                const uint32_t aV = aR + (uint32_t)sv * kAtStage + kAtKV;
                const uint32_t aPb = aP + (uint32_t)(jj & 1) * kAtPBytes;
#pragma unroll
                for (int kk = 0; kk < kAtP / 16; ++kk) {
                    const uint32_t offp = (uint32_t)(kk >> 2) * kAtQAtom + (uint32_t)(kk & 3) * 32;
                    tc::mma_f16(tmem + kAtColO, tc::desc_mn_sw128(aV + (uint32_t)kk * 2048u, kAtAtom),
                                tc::desc_k_sw128(aPb + offp), idO, (jj > 0 || kk > 0) ? 1u : 0u);
                }
                tc::mma_commit(&o_done[jj & 1]);
                tc::mma_commit(&kv_empty[sv]);
                return true;
            };
            // S_j goes ahead of P_{j-1} V_{j-1} so that it overlaps softmax j-1;
            // with a single stage tile j can only land after P_{j-1} V_{j-1}
            // has released it, so there the order is reversed.
            for (int j = 0; ok && j <= nt; ++j) {
                if (kAtStages == 1) {
                    if (j > 0) ok = issue_pv(j - 1);
                    if (ok && j < nt) ok = issue_s(j);
                } else {
                    if (j < nt) ok = issue_s(j);
                    if (ok && j > 0) ok = issue_pv(j - 1);
                }
            }
        }
        griddep_wait();
        griddep_launch_dependents();
    } else {
        // ---------------- softmax warps: thread t = position t of a tile ----------------
        const int t = threadIdx.x;
        griddep_wait();  // q is the previous kernel's output
        griddep_launch_dependents();
        trace_begin(p.trace);
        if (active) {
            for (int idx = t; idx < nh * (kAtD / 8); idx += 128) {
                const int h = idx / (kAtD / 8), c = idx - (idx / (kAtD / 8)) * (kAtD / 8);
                const uint4 qv = ldg16(p.q + (int64_t)b * p.q_sb + (int64_t)(h0 + h) * kAtD + c * 8);
                *reinterpret_cast<uint4*>(sQ + at_sw128(h, c * 8, kAtQAtom)) = qv;
            }
        }
        tc::fence_proxy_async_smem();
        tc::mbar_arrive(q_ready);
        const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
        bool ok = true;
        for (int j = 0; j < nt; ++j) {
            ok = __all_sync(0xffffffffu, tc::mbar_wait(&s_full[j & 1], (uint32_t)(j >> 1) & 1u, p.err, 75));
            if (!ok) break;
            tc::fence_after_sync();
            uint32_t v[16];
            tc::tmem_ld16(tmem + lane_base + (uint32_t)(j & 1) * 16, v);
            tc::tmem_wait_ld();
            const int pos = start + j * kAtP + t;
            const bool valid = pos < end;
            float sc[G];
#pragma unroll
            for (int h = 0; h < G; ++h) sc[h] = valid ? __uint_as_float(v[h]) * p.scale_log2 : -INFINITY;
            // per-head max over the tile's 128 positions
#pragma unroll
            for (int h = 0; h < G; ++h) {
                float mx = sc[h];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                if (lane == 0) s_red[j & 1][warp][h] = mx;
            }
            softmax_bar();
            bool resc = false;
            float mt[G];
#pragma unroll
            for (int h = 0; h < G; ++h) {
                mt[h] = fmaxf(fmaxf(s_red[j & 1][0][h], s_red[j & 1][1][h]), fmaxf(s_red[j & 1][2][h], s_red[j & 1][3][h]));
                if (h < nh) resc |= mt[h] > m_run[h] + 8.f;
            }
            float alpha[G];
#pragma unroll
            for (int h = 0; h < G; ++h) {
                const float m_use = resc ? fmaxf(m_run[h], mt[h]) : m_run[h];
                alpha[h] = m_run[h] == -INFINITY ? 0.f : at_exp2(m_run[h] - m_use);
                m_run[h] = m_use;
            }
            if (resc && j > 0) {  // uniform over the 128 threads
                const uint32_t jj = (uint32_t)(j - 1);
                ok = __all_sync(0xffffffffu, tc::mbar_wait(&o_done[jj & 1u], (jj >> 1) & 1u, p.err, 76));
                if (!ok) break;
                tc::fence_after_sync();
                uint32_t o[16];
                tc::tmem_ld16(tmem + lane_base + kAtColO, o);
                tc::tmem_wait_ld();
#pragma unroll
                for (int h = 0; h < G; ++h) o[h] = __float_as_uint(__uint_as_float(o[h]) * alpha[h]);
                tc::tmem_st16(tmem + lane_base + kAtColO, o);
                tc::tmem_wait_st();
            }
            if (j >= 2) {  // P^T buffer j & 1 is free once O += P_{j-2} V_{j-2} has completed
                ok = __all_sync(0xffffffffu,
                                tc::mbar_wait(&o_done[j & 1], (uint32_t)((j - 2) >> 1) & 1u, p.err, 77));
                if (!ok) break;
            }
            uint8_t* pb = sP + (size_t)(j & 1) * kAtPBytes;
#pragma unroll
            for (int h = 0; h < G; ++h) {
                const float pr = at_exp2(sc[h] - m_run[h]);
                l_th[h] = l_th[h] * alpha[h] + pr;
                if (h < nh) *reinterpret_cast<__half*>(pb + at_sw128(h, t, kAtQAtom)) = __float2half_rn(pr);
            }
            if (!valid) {  // rows past the end may hold anything: P = 0 there, and V must be finite
                uint8_t* vrow = ring + (size_t)(j % kAtStages) * kAtStage + kAtKV + (uint32_t)t * 128u;
#pragma unroll
                for (int a = 0; a < 2; ++a)
#pragma unroll
                    for (int q = 0; q < 8; ++q) reinterpret_cast<uint4*>(vrow + a * kAtAtom)[q] = make_uint4(0, 0, 0, 0);
            }
            tc::fence_proxy_async_smem();
            tc::fence_before_sync();
            tc::mbar_arrive(&p_full[j & 1]);
        }
        if (ok && nt > 0) {
            const uint32_t jl = (uint32_t)(nt - 1);
            ok = __all_sync(0xffffffffu, tc::mbar_wait(&o_done[jl & 1u], (jl >> 1) & 1u, p.err, 78));
            tc::fence_after_sync();
            tc::tmem_ld16(tmem + lane_base + kAtColO, o_reg);
            tc::tmem_wait_ld();
            if (!ok) {
#pragma unroll
                for (int h = 0; h < 16; ++h) o_reg[h] = 0u;
            }
        }
        // running sums: per head over the 128 threads
#pragma unroll
        for (int h = 0; h < G; ++h) {
            float ls = l_th[h];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
            if (lane == 0) s_lsum[warp][h] = ls;
        }
        softmax_bar();
#pragma unroll
        for (int h = 0; h < G; ++h) {
            if (h < nh) {
                const float Ls = (s_lsum[0][h] + s_lsum[1][h]) + (s_lsum[2][h] + s_lsum[3][h]);
                const float A = __uint_as_float(o_reg[h]);
                if (cs == 1) {
                    p.out[(int64_t)b * p.o_sb + (int64_t)(h0 + h) * kAtD + t] = __float2half_rn(Ls > 0.f ? A / Ls : 0.f);
                } else {
                    s_pa[h][t] = A;
                    if (t == 0) s_pm[h] = make_float2(m_run[h], Ls);
                }
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kAtTmemCols);
    }
    if (cs == 1) {
        trace_end(p.trace);
        return;
    }

    // ---- cluster merge: every CTA normalises a slice of the outputs
    cg::cluster_group cl = cg::this_cluster();
    cl.sync();
    if ((int)threadIdx.x < nh) {
        const int h = threadIdx.x;
        float2 pm[kAtMaxCluster];
        float M = -INFINITY;
#pragma unroll
        for (int r = 0; r < kAtMaxCluster; ++r) {
            pm[r] = r < cs ? *cl.map_shared_rank(&s_pm[h], r) : make_float2(-INFINITY, 0.f);
            M = fmaxf(M, pm[r].x);
        }
        float Ls = 0.f;
#pragma unroll
        for (int r = 0; r < kAtMaxCluster; ++r) {
            pm[r].x = pm[r].x == -INFINITY ? 0.f : exp2f(pm[r].x - M);
            Ls = fmaf(pm[r].y, pm[r].x, Ls);
        }
        const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
#pragma unroll
        for (int r = 0; r < kAtMaxCluster; ++r) s_wt[h][r] = pm[r].x * inv;
    }
    __syncthreads();
    for (int idx = split * (int)blockDim.x + threadIdx.x; idx < nh * kAtD; idx += cs * (int)blockDim.x) {
        const int h = idx / kAtD, d = idx - (idx / kAtD) * kAtD;
        // all ranks' partials requested at once (one distributed-shared-memory
        // round trip), then summed in rank order
        float part[kAtMaxCluster];
#pragma unroll
        for (int r = 0; r < kAtMaxCluster; ++r) part[r] = r < cs ? *cl.map_shared_rank(&s_pa[h][d], r) : 0.f;
        float A = 0.f;
#pragma unroll
        for (int r = 0; r < kAtMaxCluster; ++r)
            if (r < cs) A = fmaf(part[r], s_wt[h][r], A);
        p.out[(int64_t)b * p.o_sb + (int64_t)(h0 + h) * kAtD + d] = __float2half_rn(A);
    }
    cl.sync();
    trace_end(p.trace);
}

// Cluster size for the tensor-core kernel: about one CTA per SM over the
// batch's (sequence, kv head group) pairs, at most 8, at least one tile each.
static int attn_tc_splits(int batch, int nkv, int hg, int max_len) {
    const long ctas1 = (long)batch * nkv * hg;
    long cs = sm_count() / ctas1;
    const long by_len = (max_len + kAtP - 1) / kAtP;
    if (cs > by_len) cs = by_len;
    if (cs > kAtMaxCluster) cs = kAtMaxCluster;
    if (cs < 1) cs = 1;
    return (int)cs;
}

template <int G, int STAGES>
static int launch_tc_g(const CUtensorMap& tk, const CUtensorMap& tv, const AttnTcParams& p, int cs, int B,
                       cudaStream_t s, bool pdl) {
    auto kern = attn_tc_kernel<G, STAGES>;
    constexpr size_t smem = AtSmem<STAGES>::BYTES;
    B2_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid((unsigned)cs, (unsigned)(p.nkv * p.hg), (unsigned)B);
    B2_TRY(launch_cluster(kern, grid, dim3(192), smem, s, pdl, (unsigned)cs, tk, tv, p));
    return B2_OK;
}

bool attn_tc_enabled() {
    static int on = -1;
    if (on < 0) {
        const char* e = getenv("B2_ATTN_TC");
        on = (e && e[0] == '0') ? 0 : 1;
    }
    return on == 1;
}

// Tensor-core launch (head_dim 128, group <= 8 per head group); the
// arguments are those of attn_cl_launch.  B2_ERR_UNSUPPORTED when the shape
// does not fit.
int attn_tc_launch(const __half* q, int64_t q_sb, __half* out, int64_t o_sb, const __half* k, const __half* v,
                   int64_t sb, int64_t sh, int64_t ss, int max_len, const int* seq_lens, int len_const, int B,
                   int nq, int nkv, int D, int early_kv, int lean, TraceSlot trace, cudaStream_t s, bool pdl) {
    if (!attn_tc_enabled() || D != kAtD || max_len < 1 || B < 1 || B > 65535) return B2_ERR_UNSUPPORTED;
    if (!aligned16(k) || !aligned16(v) || !aligned16(q) || (q_sb & 7) || (sb & 7) || (sh & 7) || (ss & 7) ||
        sh <= 0 || ss <= 0 || sb < 0)
        return B2_ERR_UNSUPPORTED;
    int* err = wait_error_word();
    if (!err) return B2_ERR_STATE;
    const int group = nq / nkv;
    const int G = group <= 4 ? 4 : 8;
    AttnTcParams p = {};
    p.q = q;
    p.q_sb = q_sb;
    p.out = out;
    p.o_sb = o_sb;
    p.seq_lens = seq_lens;
    p.len_const = len_const;
    p.nq = nq;
    p.nkv = nkv;
    p.group = group;
    p.hg = (group + G - 1) / G;
    p.scale_log2 = 1.4426950408889634f / sqrtf((float)D);
    p.early_kv = early_kv;
    p.kp = k;
    p.vp = v;
    p.sb = sb;
    p.sh = sh;
    p.ss = ss;
    p.err = err;
    p.trace = trace;
    const bool head_inner = sh < ss;
    p.head_inner = head_inner ? 1 : 0;
    uint64_t dims[4], st[3];
    uint32_t box[4];
    dims[0] = (uint64_t)D;
    box[0] = 64;
    if (head_inner) {
        dims[1] = (uint64_t)nkv; st[0] = (uint64_t)sh * 2; box[1] = 1;
        dims[2] = (uint64_t)max_len; st[1] = (uint64_t)ss * 2; box[2] = kAtP;
    } else {
        dims[1] = (uint64_t)max_len; st[0] = (uint64_t)ss * 2; box[1] = kAtP;
        dims[2] = (uint64_t)nkv; st[1] = (uint64_t)sh * 2; box[2] = 1;
    }
    dims[3] = (uint64_t)B;
    st[2] = sb > 0 ? (uint64_t)sb * 2 : st[1] * dims[2];
    box[3] = 1;
    CUtensorMap tk, tv;
    int rc = make_tensor_map(&tk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, k, dims, st, box);
    if (rc != B2_OK) return rc;
    rc = make_tensor_map(&tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, v, dims, st, box);
    if (rc != B2_OK) return rc;
    const int cs = attn_tc_splits(B, nkv, p.hg, max_len);
    // Ring depth: 3 stages (210 KB of shared memory) by default; `lean`
    // callers run register-streaming GEMVs around the attention, whose
    // in-flight loads need the SM's L1, and an SM configured for 210 KB of
    // shared memory keeps only ~28 KB of it: they get 2 stages (~146 KB),
    // or 1 when no split can hold more than one tile.
    // More CTAs than SMs (many sequences) at moderate context: a 1-stage
    // ring (76 KB) lets two or three CTAs share an SM, so the grid runs as
    // one wave instead of 1.7 waves of one CTA per SM (batch 32, ctx 512:
    // 24.6 vs 28.7 us).  Long contexts keep the deeper ring (ctx 32K: 638
    // vs 692 us).
    const long ctas = (long)cs * B * nkv * p.hg;
    const bool many = ctas > sm_count() && max_len <= 8192;
    const int stages = many ? 1 : (!lean ? 3 : ((max_len + cs - 1) / cs <= kAtP ? 1 : 2));
    if (G == 4) {
        if (stages == 1) return launch_tc_g<4, 1>(tk, tv, p, cs, B, s, pdl);
        if (stages == 2) return launch_tc_g<4, 2>(tk, tv, p, cs, B, s, pdl);
        return launch_tc_g<4, 3>(tk, tv, p, cs, B, s, pdl);
    }
    if (stages == 1) return launch_tc_g<8, 1>(tk, tv, p, cs, B, s, pdl);
    if (stages == 2) return launch_tc_g<8, 2>(tk, tv, p, cs, B, s, pdl);
    return launch_tc_g<8, 3>(tk, tv, p, cs, B, s, pdl);
}

// Paged form: K / V pools [num_blocks][bs][nkv][128], block tables [B][maxb]
// (bs a multiple of 8 dividing 128), sequence lengths seq_lens[B] <=
// max_len.  Same kernel; the producer fetches each 128-position tile as
// 128/bs block boxes.
int attn_tc_launch_paged(const __half* q, int64_t q_sb, __half* out, int64_t o_sb, const __half* kpool,
                         const __half* vpool, int num_blocks, int bs, const int* bt, int maxb, int max_len,
                         const int* seq_lens, int B, int nq, int nkv, int D, int early_kv, int lean, TraceSlot trace,
                         cudaStream_t s, bool pdl) {
    if (D != kAtD || max_len < 1 || B < 1 || B > 65535 || num_blocks < 1 || maxb < 1 || !bt) return B2_ERR_UNSUPPORTED;
    if (bs < 8 || (bs & 7) || kAtP % bs) return B2_ERR_UNSUPPORTED;
    if (!aligned16(kpool) || !aligned16(vpool) || !aligned16(q) || (q_sb & 7)) return B2_ERR_UNSUPPORTED;
    int* err = wait_error_word();
    if (!err) return B2_ERR_STATE;
    const int group = nq / nkv;
    const int G = group <= 4 ? 4 : 8;
    AttnTcParams p = {};
    p.q = q;
    p.q_sb = q_sb;
    p.out = out;
    p.o_sb = o_sb;
    p.seq_lens = seq_lens;
    p.nq = nq;
    p.nkv = nkv;
    p.group = group;
    p.hg = (group + G - 1) / G;
    p.scale_log2 = 1.4426950408889634f / sqrtf((float)D);
    p.early_kv = early_kv;
    p.kp = kpool;
    p.vp = vpool;
    p.bt = bt;
    p.maxb = maxb;
    p.bs = bs;
    p.err = err;
    p.trace = trace;
    // (128 columns, head, slot, block): box 64 x 1 x bs x 1
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)nkv, (uint64_t)bs, (uint64_t)num_blocks};
    const uint64_t st[3] = {(uint64_t)D * 2, (uint64_t)nkv * D * 2, (uint64_t)bs * nkv * D * 2};
    const uint32_t box[4] = {64u, 1u, (uint32_t)bs, 1u};
    CUtensorMap tk, tv;
    int rc = make_tensor_map(&tk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, kpool, dims, st, box);
    if (rc != B2_OK) return rc;
    rc = make_tensor_map(&tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, vpool, dims, st, box);
    if (rc != B2_OK) return rc;
    const int cs = attn_tc_splits(B, nkv, p.hg, max_len);
    const long ctas = (long)cs * B * nkv * p.hg;
    const bool many = ctas > sm_count() && max_len <= 8192;
    const int stages = many ? 1 : (!lean ? 3 : ((max_len + cs - 1) / cs <= kAtP ? 1 : 2));
    if (G == 4) {
        if (stages == 1) return launch_tc_g<4, 1>(tk, tv, p, cs, B, s, pdl);
        if (stages == 2) return launch_tc_g<4, 2>(tk, tv, p, cs, B, s, pdl);
        return launch_tc_g<4, 3>(tk, tv, p, cs, B, s, pdl);
    }
    if (stages == 1) return launch_tc_g<8, 1>(tk, tv, p, cs, B, s, pdl);
    if (stages == 2) return launch_tc_g<8, 2>(tk, tv, p, cs, B, s, pdl);
    return launch_tc_g<8, 3>(tk, tv, p, cs, B, s, pdl);
}

}  // namespace b2
