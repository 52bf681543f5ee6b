// attention_cl.cu -- split-KV GQA decode attention with TMA-fed K/V tiles and
// the split merge inside a thread-block cluster, sm_100a.
//
// One cluster per (sequence, kv head x head group); its CS CTAs (CS <= 8,
// fixed on the host from max_seq_len so a captured graph stays valid) take
// consecutive position chunks of that kv head and stream them ONCE for all
// the group's query heads (GQA).  Per CTA:
//   warp 4, lane 0   TMA producer: K and V tiles of P positions (P x D fp16
//                    rows, one 4-D tensor map over the cache view, so any
//                    (batch, head, position) strides work) into a ring of
//                    stages with full / empty mbarriers.  In the decode step
//                    the tiles holding only rows older than the newest
//                    position go out before the programmatic-launch wait
//                    (those rows were written by earlier steps);
//   warps 0..3       each owns 1/4 of every tile: LP = D/8 lanes per
//                    position, a lane holding one 16-byte chunk of the K row
//                    and of the V row, q pre-scaled by log2(e)/sqrt(D),
//                    online softmax per query head, accumulators in registers.
// The four warps merge in shared memory; the CTA's partial (max, sum and the
// unnormalised output of each head) stays in its shared memory, and after a
// cluster barrier every CTA merges a slice of the outputs by reading all CS
// partials through distributed shared memory (same order everywhere, so the
// result does not depend on timing).  No global scratch, no arrival counter,
// no second kernel.  Every mbarrier wait is bounded (tc.cuh).
// Reference replaced: src/cuda/decode_attention_split.cu:28-214 and
// src/cuda/decode_attention.cu:15-141.
#include <cmath>
#include <cstdlib>

#include <cooperative_groups.h>

#include "attention.cuh"
#include "tc.cuh"

namespace cg = cooperative_groups;

namespace b2 {

struct AttnClParams {
    const __half* q;
    int64_t q_sb;  // elements between sequences of q (heads D apart)
    __half* out;
    int64_t o_sb;
    const int* seq_lens;  // null: every sequence has len_const positions
    int len_const;
    int nq, nkv, group, hg;
    float scale_log2;
    int early_kv;    // decode step: rows older than the newest may be read before the PDL wait
    int head_inner;  // tensor map dims are {D, head, pos, batch} (else {D, pos, head, batch})
    int stages;
    int* err;
    TraceSlot trace;
};

constexpr int kClWarps = 4;                 // consumer warps
constexpr int kClThreads = kClWarps * 32 + 32;  // + the producer warp
constexpr int kClMaxCluster = 8;

template <int D, int G>
struct ClGeom {
    static constexpr int C8 = D / 8;                     // 16-byte chunks per row
    static constexpr int LP = C8;                        // lanes per position
    static constexpr int PPW = 32 / LP;                  // positions per warp step
    static constexpr int UNR = G <= 4 ? 4 : 2;           // warp steps per tile
    static constexpr int WT = PPW * UNR;                 // positions per warp per tile
    static constexpr int P = kClWarps * WT;              // positions per tile
    static constexpr uint32_t ROW = D * 2;               // bytes per K or V row
    static constexpr uint32_t KV_BYTES = P * ROW;        // one K (or V) tile
    static constexpr uint32_t STAGE = 2 * KV_BYTES;
};

template <int D, int G>
__global__ void __launch_bounds__(kClThreads) attn_cl_kernel(const __grid_constant__ CUtensorMap tmK,
                                                             const __grid_constant__ CUtensorMap tmV,
                                                             const AttnClParams p) {
    using Geo = ClGeom<D, G>;
    constexpr int LP = Geo::LP, PPW = Geo::PPW, UNR = Geo::UNR, P = Geo::P;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    const int stages = p.stages;
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + (size_t)stages * Geo::STAGE);
    uint64_t* empty = full + stages;
    __shared__ float s_m[kClWarps][G], s_l[kClWarps][G];
    __shared__ __align__(16) float s_acc[kClWarps][G][D];
    __shared__ float2 s_pm[G];             // this CTA's (max, sum) per head
    __shared__ __align__(16) float s_pa[G][D];  // this CTA's unnormalised output per head
    __shared__ float s_wt[G][kClMaxCluster];

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int cs = (int)gridDim.x;  // cluster size = splits
    const int split = blockIdx.x;
    const int kvh = blockIdx.y / p.hg, hgi = blockIdx.y - (blockIdx.y / p.hg) * p.hg;
    const int b = blockIdx.z;
    const int h0 = kvh * p.group + hgi * G;
    const int nh = min(G, p.group - hgi * G);

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], kClWarps);
        }
        tc::fence_barrier_init();
    }
    __syncthreads();
    if (!p.early_kv) griddep_wait();

    const int L = p.seq_lens ? p.seq_lens[b] : p.len_const;
    int chunk = (L + cs - 1) / cs;
    chunk = ((chunk + P - 1) / P) * P;
    if (chunk < P) chunk = P;
    const int n_used = L > 0 ? (L + chunk - 1) / chunk : 0;
    const bool active = split < n_used;
    const int start = split * chunk;
    const int end = active ? min(L, start + chunk) : start;
    const int nt = active ? (end - start + P - 1) / P : 0;

    float m_run[G], l_run[G], acc[G][8];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m_run[g] = -INFINITY;
        l_run[g] = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[g][j] = 0.f;
    }

    if (warp == kClWarps) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            bool waited = !p.early_kv;
            for (int i = 0; i < nt; ++i) {
                const int s = i % stages;
                if (i >= stages && !tc::mbar_wait(&empty[s], (uint32_t)((i / stages) - 1) & 1u, p.err, 61)) break;
                const int pos0 = start + i * P;
                if (!waited && pos0 + P > L - 1) {  // this tile holds the newest row
                    griddep_wait();
                    waited = true;
                }
                uint8_t* st = ring + (size_t)s * Geo::STAGE;
                tc::mbar_arrive_expect_tx(&full[s], Geo::STAGE);
                if (p.head_inner) {
                    tc::tma_load_4d(st, &tmK, &full[s], 0, kvh, pos0, b);
                    tc::tma_load_4d(st + Geo::KV_BYTES, &tmV, &full[s], 0, kvh, pos0, b);
                } else {
                    tc::tma_load_4d(st, &tmK, &full[s], 0, pos0, kvh, b);
                    tc::tma_load_4d(st + Geo::KV_BYTES, &tmV, &full[s], 0, pos0, kvh, b);
                }
            }
        }
        griddep_wait();
        griddep_launch_dependents();
    } else {
        // ---------------- consumers ----------------
        griddep_wait();  // q is the previous kernel's output
        griddep_launch_dependents();
        trace_begin(p.trace);
        const int pidx = lane / LP, c = lane - (lane / LP) * LP;
        float qf[G][8];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            if (g < nh && active) {
                const uint4 qv = ldg16(p.q + (int64_t)b * p.q_sb + (int64_t)(h0 + g) * D + c * 8);
                unpack8(qv, qf[g]);
#pragma unroll
                for (int j = 0; j < 8; ++j) qf[g][j] *= p.scale_log2;
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) qf[g][j] = 0.f;
            }
        }
        for (int i = 0; i < nt; ++i) {
            const int s = i % stages;
            const bool ok = __all_sync(0xffffffffu, tc::mbar_wait(&full[s], (uint32_t)(i / stages) & 1u, p.err, 62));
            if (!ok) break;
            const uint8_t* st = ring + (size_t)s * Geo::STAGE;
            const int base = start + i * P + warp * Geo::WT;
            uint4 kr[UNR], vr[UNR];
            bool valid[UNR];
#pragma unroll
            for (int u = 0; u < UNR; ++u) {
                const int r = warp * Geo::WT + u * PPW + pidx;  // row inside the tile
                valid[u] = base + u * PPW + pidx < end;
                kr[u] = *reinterpret_cast<const uint4*>(st + r * Geo::ROW + c * 16);
                vr[u] = *reinterpret_cast<const uint4*>(st + Geo::KV_BYTES + r * Geo::ROW + c * 16);
                if (!valid[u]) vr[u] = make_uint4(0, 0, 0, 0);  // rows past the end may hold anything
            }
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&empty[s]);
            float sc[UNR][G];
#pragma unroll
            for (int u = 0; u < UNR; ++u) {
                float kf[8];
                unpack8(kr[u], kf);
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    float d = 0.f;
#pragma unroll
                    for (int j = 0; j < 8; ++j) d = fmaf(qf[g][j], kf[j], d);
#pragma unroll
                    for (int o = 1; o < LP; o <<= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
                    sc[u][g] = valid[u] ? d : -INFINITY;
                }
            }
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float mt = sc[0][g];
#pragma unroll
                for (int u = 1; u < UNR; ++u) mt = fmaxf(mt, sc[u][g]);
#pragma unroll
                for (int o = LP; o < 32; o <<= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
                const float m_new = fmaxf(m_run[g], mt);
                if (m_new == -INFINITY) continue;  // nothing valid yet in this warp
                const float alpha = exp2f(m_run[g] - m_new);
                l_run[g] *= alpha;
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[g][j] *= alpha;
#pragma unroll
                for (int u = 0; u < UNR; ++u) {
                    const float pr = exp2f(sc[u][g] - m_new);
                    l_run[g] += pr;
                    float vf[8];
                    unpack8(vr[u], vf);
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc[g][j] = fmaf(pr, vf[j], acc[g][j]);
                }
                m_run[g] = m_new;
            }
        }
        // merge the PPW position groups of the warp (the running max is warp-uniform)
#pragma unroll
        for (int g = 0; g < G; ++g) {
#pragma unroll
            for (int o = LP; o < 32; o <<= 1) {
                l_run[g] += __shfl_xor_sync(0xffffffffu, l_run[g], o);
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[g][j] += __shfl_xor_sync(0xffffffffu, acc[g][j], o);
            }
        }
        if (pidx == 0) {
#pragma unroll
            for (int g = 0; g < G; ++g)
#pragma unroll
                for (int j = 0; j < 8; ++j) s_acc[warp][g][c * 8 + j] = acc[g][j];
        }
        if (lane == 0) {
#pragma unroll
            for (int g = 0; g < G; ++g) {
                s_m[warp][g] = m_run[g];
                s_l[warp][g] = l_run[g];
            }
        }
    }
    __syncthreads();

    // ---- this CTA's partial: the four warps merged
    for (int idx = threadIdx.x; idx < nh * D; idx += kClThreads) {
        const int g = idx / D, d = idx - (idx / D) * D;
        float M = s_m[0][g];
#pragma unroll
        for (int w = 1; w < kClWarps; ++w) M = fmaxf(M, s_m[w][g]);
        float Ls = 0.f, A = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kClWarps; ++w) {
                const float sc = s_m[w][g] == -INFINITY ? 0.f : exp2f(s_m[w][g] - M);
                Ls = fmaf(s_l[w][g], sc, Ls);
                A = fmaf(s_acc[w][g][d], sc, A);
            }
        }
        if (cs == 1) {
            p.out[(int64_t)b * p.o_sb + (int64_t)(h0 + g) * D + d] = __float2half_rn(Ls > 0.f ? A / Ls : 0.f);
        } else {
            s_pa[g][d] = A;
            if (d == 0) s_pm[g] = make_float2(M, Ls);
        }
    }
    if (cs == 1) {
        __syncthreads();
        trace_end(p.trace);
        return;
    }

    // ---- cluster merge: every CTA normalises a slice of the outputs
    cg::cluster_group cl = cg::this_cluster();
    cl.sync();
    if ((int)threadIdx.x < nh) {
        const int g = threadIdx.x;
        float2 pm[kClMaxCluster];
        float M = -INFINITY;
#pragma unroll
        for (int r = 0; r < kClMaxCluster; ++r) {
            pm[r] = r < cs ? *cl.map_shared_rank(&s_pm[g], r) : make_float2(-INFINITY, 0.f);
            M = fmaxf(M, pm[r].x);
        }
        float Ls = 0.f;
#pragma unroll
        for (int r = 0; r < kClMaxCluster; ++r) {
            pm[r].x = pm[r].x == -INFINITY ? 0.f : exp2f(pm[r].x - M);
            Ls = fmaf(pm[r].y, pm[r].x, Ls);
        }
        const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
#pragma unroll
        for (int r = 0; r < kClMaxCluster; ++r) s_wt[g][r] = pm[r].x * inv;
    }
    __syncthreads();
    for (int idx = split * kClThreads + threadIdx.x; idx < nh * D; idx += cs * kClThreads) {
        const int g = idx / D, d = idx - (idx / D) * D;
        // all ranks' partials requested at once, then summed in rank order
        float part[kClMaxCluster];
#pragma unroll
        for (int r = 0; r < kClMaxCluster; ++r) part[r] = r < cs ? *cl.map_shared_rank(&s_pa[g][d], r) : 0.f;
        float A = 0.f;
#pragma unroll
        for (int r = 0; r < kClMaxCluster; ++r)
            if (r < cs) A = fmaf(part[r], s_wt[g][r], A);
        p.out[(int64_t)b * p.o_sb + (int64_t)(h0 + g) * D + d] = __float2half_rn(A);
    }
    cl.sync();  // no CTA leaves while a peer still reads its partial
    trace_end(p.trace);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct AttnClShape {
    const __half* k;
    const __half* v;
    int64_t sb, sh, ss;  // element strides of the cache views (d stride 1)
    int max_len;         // positions the views cover (tensor-map extent)
    int batch, nq, nkv, D;
};

template <int D, int G>
static int launch_cl_dg(const AttnClShape& sh, AttnClParams p, int cs, cudaStream_t s, bool pdl) {
    using Geo = ClGeom<D, G>;
    CUtensorMap tk, tv;
    const bool head_inner = sh.sh < sh.ss;
    p.head_inner = head_inner ? 1 : 0;
    uint64_t dims[4], st[3];
    uint32_t box[4];
    dims[0] = (uint64_t)D;
    box[0] = (uint32_t)D;
    if (head_inner) {
        dims[1] = (uint64_t)sh.nkv; st[0] = (uint64_t)sh.sh * 2; box[1] = 1;
        dims[2] = (uint64_t)sh.max_len; st[1] = (uint64_t)sh.ss * 2; box[2] = (uint32_t)Geo::P;
    } else {
        dims[1] = (uint64_t)sh.max_len; st[0] = (uint64_t)sh.ss * 2; box[1] = (uint32_t)Geo::P;
        dims[2] = (uint64_t)sh.nkv; st[1] = (uint64_t)sh.sh * 2; box[2] = 1;
    }
    dims[3] = (uint64_t)sh.batch;
    st[2] = sh.sb > 0 ? (uint64_t)sh.sb * 2 : st[1] * dims[2];  // sb = 0: one sequence, any legal stride
    box[3] = 1;
    int rc = make_tensor_map_plain(&tk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, sh.k, dims, st, box);
    if (rc != B2_OK) return rc;
    rc = make_tensor_map_plain(&tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, sh.v, dims, st, box);
    if (rc != B2_OK) return rc;
    const size_t smem = (size_t)p.stages * Geo::STAGE + 2 * (size_t)p.stages * 8 + 128;
    auto kern = attn_cl_kernel<D, G>;
    B2_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid((unsigned)cs, (unsigned)(sh.nkv * p.hg), (unsigned)sh.batch);
    B2_TRY(launch_cluster(kern, grid, dim3(kClThreads), smem, s, pdl, (unsigned)cs, tk, tv, p));
    return B2_OK;
}

template <int D>
static int launch_cl_d(const AttnClShape& sh, const AttnClParams& p, int G, int cs, cudaStream_t s, bool pdl) {
    switch (G) {
        case 1: return launch_cl_dg<D, 1>(sh, p, cs, s, pdl);
        case 2: return launch_cl_dg<D, 2>(sh, p, cs, s, pdl);
        case 4: return launch_cl_dg<D, 4>(sh, p, cs, s, pdl);
        default: return launch_cl_dg<D, 8>(sh, p, cs, s, pdl);
    }
}

// B2_ATTN_CLUSTER=0 in the environment selects the global-merge kernel
// (attention.cu) everywhere instead.
static bool attn_cl_enabled() {
    static int on = -1;
    if (on < 0) {
        const char* e = getenv("B2_ATTN_CLUSTER");
        on = (e && e[0] == '0') ? 0 : 1;
    }
    return on == 1;
}

bool attn_cl_supported(int D, int64_t sb, int64_t sh, int64_t ss, const void* k, const void* v) {
    if (!attn_cl_enabled()) return false;
    if (D != 32 && D != 64 && D != 128 && D != 256) return false;
    if (!aligned16(k) || !aligned16(v)) return false;
    if ((sb & 7) || (sh & 7) || (ss & 7) || sh <= 0 || ss <= 0 || sb < 0) return false;
    return true;
}

// Cluster size (splits per (sequence, kv head group)) for `batch` sequences
// of at most max_len positions: about two CTAs per SM, at most 8, at least
// one tile of positions per split.
int attn_cl_splits(int batch, int nq, int nkv, int D, int max_len) {
    const int group = nq / nkv;
    const int G = group <= 1 ? 1 : (group <= 2 ? 2 : (group <= 4 ? 4 : 8));
    const long ctas1 = (long)batch * nkv * ((group + G - 1) / G);
    long cs = (2L * sm_count() + ctas1 - 1) / ctas1;
    const int P = kClWarps * (32 / (D / 8)) * (G <= 4 ? 4 : 2);
    const long by_len = (max_len + P - 1) / P;
    if (cs > by_len) cs = by_len;
    if (cs > kClMaxCluster) cs = kClMaxCluster;
    if (cs < 1) cs = 1;
    return (int)cs;
}

// Launch: q [B] rows q_sb apart, out [B] rows o_sb apart, K/V views
// (sb, sh, ss) covering max_len positions.  head_dim 128 runs on the tensor
// cores (attention_tc.cu), other head dims on this file's kernel.
// B2_ERR_UNSUPPORTED when the shape fits neither (the caller then uses
// attn_decode_launch).
int attn_cl_launch(const __half* q, int64_t q_sb, __half* out, int64_t o_sb, const __half* k, const __half* v,
                   int64_t sb, int64_t sh, int64_t ss, int max_len, const int* seq_lens, int len_const, int B,
                   int nq, int nkv, int D, int early_kv, int lean, TraceSlot trace, cudaStream_t s, bool pdl) {
    if (attn_cl_enabled()) {  // head_dim 128: the tensor-core form (attention_tc.cu)
        const int rc = attn_tc_launch(q, q_sb, out, o_sb, k, v, sb, sh, ss, max_len, seq_lens, len_const, B, nq, nkv,
                                      D, early_kv, lean, trace, s, pdl);
        if (rc != B2_ERR_UNSUPPORTED) return rc;
    }
    if (!attn_cl_supported(D, sb, sh, ss, k, v) || max_len < 1 || B < 1 || B > 65535) return B2_ERR_UNSUPPORTED;
    // Long streams (more than 8192 positions per kv head over the batch) run
    // faster on the global-merge kernel's many small CTAs: this kernel's four
    // consumer warps per CTA are bound by their per-position arithmetic there.
    if ((int64_t)B * max_len > 8192) return B2_ERR_UNSUPPORTED;
    if (!aligned16(q) || (q_sb & 7)) return B2_ERR_UNSUPPORTED;
    int* err = wait_error_word();
    if (!err) return B2_ERR_STATE;
    const int group = nq / nkv;
    const int G = group <= 1 ? 1 : (group <= 2 ? 2 : (group <= 4 ? 4 : 8));
    AttnClParams p = {};
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
    p.err = err;
    p.trace = trace;
    const int cs = attn_cl_splits(B, nq, nkv, D, max_len);
    const long ctas = (long)cs * B * nkv * p.hg;
    p.stages = ctas <= sm_count() ? 8 : 4;
    AttnClShape shp{k, v, sb, sh, ss, max_len, B, nq, nkv, D};
    switch (D) {
        case 32: return launch_cl_d<32>(shp, p, G, cs, s, pdl);
        case 64: return launch_cl_d<64>(shp, p, G, cs, s, pdl);
        case 128: return launch_cl_d<128>(shp, p, G, cs, s, pdl);
        default: return launch_cl_d<256>(shp, p, G, cs, s, pdl);
    }
}

}  // namespace b2
