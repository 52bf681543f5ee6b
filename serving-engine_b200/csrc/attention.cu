// attention.cu -- split-KV GQA decode attention with an in-kernel LSE merge, sm_100a.
//
// One CTA streams one contiguous split of the positions of one
// (sequence, kv head) ONCE for all of that kv head's query heads (GQA
// grouping: K/V bytes cross HBM once per kv head, not once per q head).
// Inside the CTA each warp owns a strided subset of position tiles; a warp
// covers PPW positions per step with LP = D/8 lanes per position, each lane
// holding one 16-byte chunk of K and of V, so a K or V row is read as one
// fully coalesced 16*LP-byte segment.  Scores live in the log2 domain (q is
// pre-scaled by log2(e)/sqrt(D)); the softmax is online (running max,
// rescaled sum and accumulator per query head).  Each split writes an
// unnormalised partial output plus its (max, sum) pair, and the splits are
// merged as described below.  With one split the CTA writes the final output
// directly and needs no scratch.
//
// The grid carries the maximum split count, fixed on the host from
// max_seq_len (so a captured graph stays valid as the context grows); each
// CTA derives the live split count from seq_lens[b] on the device (a split
// covers at least one iteration of all its warps) and idle splits exit at
// once.  The splits of one (sequence, kv head) are merged by whichever CTA
// finishes last: every CTA publishes its partial, fences, and bumps a
// per-(sequence, kv head) counter; the CTA that sees the final count stages
// the normalised split weights in shared memory, sums the partials from L2
// with independent loads and resets the counter to zero, so no second kernel
// is launched.
//
// In the decode step each warp requests its first tile of K/V rows older
// than the newest position before it waits on the q|k|v kernel that precedes
// it (those rows were written by earlier steps), so that DRAM latency
// overlaps the previous kernel's tail.
//
// Reference replaced: src/cuda/decode_attention_split.cu:28-214 (one CTA per
// (q head, sequence), head_dim fixed at 64, no split and no combine) and
// src/cuda/decode_attention.cu:15-141 (serial per-token loop).
#include <cmath>

#include "attention.cuh"
#include "common.cuh"

namespace b2 {

struct AttnParams {
    const __half* q;
    int64_t q_sb;  // element stride between sequences of q (heads are D apart)
    const __half* k;
    const __half* v;
    int64_t sb, sh, ss;  // K/V view strides in elements (d stride 1)
    const int* seq_lens;
    int causal_base;  // >= 0: seq_len(b) = causal_base + b + 1 (prefill use)
    int len_const;    // > 0 and seq_lens == null: every sequence has this length
    __half* out;
    int64_t o_sb;
    float* part;    // [B][nq][splits][D]
    float2* ml;     // [B][nq][splits] (max, sum)
    int* counters;  // [B][nkv*hg] arrival counts, zero between launches
    int splits;     // maximum splits (grid.x)
    int nq, nkv, group, hg;
    float scale_log2;
    // Decode-step form only: seq_lens and every K/V row except the newest
    // (position seq_len - 1, written by the kernel just before) were written
    // at least two kernels earlier, so they may be read before the
    // programmatic-launch wait.
    int early_kv;
    TraceSlot trace;
};

constexpr int kAttnWarps = 4;
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr int kMaxSplits = 128;

// 16-byte asynchronous global->shared copy (zero-filled when !valid);
// completion tracked per thread with commit / wait groups.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
    const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sa), "l"(gmem), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

constexpr int kAttnStages = 3;  // K/V tiles each lane keeps in flight (cp.async ring)

template <int C8>
struct LaneMap {
    static constexpr int LP = C8 <= 2 ? 2 : (C8 <= 4 ? 4 : (C8 <= 8 ? 8 : (C8 <= 16 ? 16 : 32)));
    static constexpr int PPW = 32 / LP;
};

template <int D, int G>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const AttnParams p) {
    constexpr int C8 = D / 8;
    constexpr int LP = LaneMap<C8>::LP;
    constexpr int PPW = LaneMap<C8>::PPW;
    constexpr int UNR = G <= 4 ? 4 : 2;
    constexpr int WT = PPW * UNR;             // positions one warp covers per iteration
    constexpr int kMinChunk = kAttnWarps * WT;  // a split is at least one CTA iteration
    __shared__ float s_m[kAttnWarps][G], s_l[kAttnWarps][G];
    __shared__ __align__(16) float s_acc[kAttnWarps][G][D];
    __shared__ float s_w[G][kMaxSplits];

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int split = blockIdx.x;
    const int kvh = blockIdx.y / p.hg, hgi = blockIdx.y - (blockIdx.y / p.hg) * p.hg;
    const int b = blockIdx.z;
    const int h0 = kvh * p.group + hgi * G;
    const int nh = min(G, p.group - hgi * G);
    const int pidx = lane / LP, c = lane - (lane / LP) * LP;
    const bool cact = c < C8;

    if (!p.early_kv) {
        griddep_wait();
        griddep_launch_dependents();
        trace_begin(p.trace);
    }

    const int L = p.causal_base >= 0 ? p.causal_base + b + 1 : (p.seq_lens ? p.seq_lens[b] : p.len_const);
    int chunk = (L + p.splits - 1) / p.splits;
    chunk = max(chunk, kMinChunk);
    const int n_used = L > 0 ? (L + chunk - 1) / chunk : 1;
    if (split >= n_used) {  // idle split at this context length
        if (p.early_kv) griddep_launch_dependents();
        return;
    }
    const int start = split * chunk;
    const int end = min(L, start + chunk);

    const __half* kb = p.k + (int64_t)b * p.sb + (int64_t)kvh * p.sh + c * 8;
    const __half* vb = p.v + (int64_t)b * p.sb + (int64_t)kvh * p.sh + c * 8;

    // K/V tiles stream through a per-lane cp.async ring (each lane copies and
    // later reads only its own 16-byte slots), kAttnStages - 1 tiles ahead of
    // the one being computed.  In the decode-step form the first tiles are
    // requested before waiting on the previous kernel, without the newest row
    // (written by that kernel), which is read directly once the wait is over.
    extern __shared__ __align__(16) uint4 kv_ring[];  // [warp][stage][UNR][K,V][lane]
    uint4* ring = kv_ring + (size_t)warp * kAttnStages * UNR * 2 * 32;
    const int tile0 = start + warp * WT;
    const int nt = tile0 < end ? (end - tile0 + kAttnWarps * WT - 1) / (kAttnWarps * WT) : 0;
    auto issue = [&](int i, int lim) {
        if (i < nt) {
            const int tb = tile0 + i * kAttnWarps * WT;
            uint4* st = ring + (size_t)(i % kAttnStages) * UNR * 2 * 32;
#pragma unroll
            for (int u = 0; u < UNR; ++u) {
                const int pos = tb + u * PPW + pidx;
                const bool ok = cact && pos < lim;
                const int64_t off = ok ? (int64_t)pos * p.ss : 0;
                cp_async16(st + (u * 2 + 0) * 32 + lane, kb + off, ok);
                cp_async16(st + (u * 2 + 1) * 32 + lane, vb + off, ok);
            }
        }
        cp_async_commit();
    };
    {
        const int lim = p.early_kv ? min(end, L - 1) : end;
#pragma unroll
        for (int i = 0; i < kAttnStages - 1; ++i) issue(i, lim);
    }
    if (p.early_kv) {
        griddep_wait();
        griddep_launch_dependents();
        trace_begin(p.trace);
    }

    float qf[G][8];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        if (g < nh && cact) {
            const uint4 qv = ldg16(p.q + (int64_t)b * p.q_sb + (int64_t)(h0 + g) * D + c * 8);
            unpack8(qv, qf[g]);
#pragma unroll
            for (int j = 0; j < 8; ++j) qf[g][j] *= p.scale_log2;
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) qf[g][j] = 0.f;
        }
    }

    float m_run[G], l_run[G], acc[G][8];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m_run[g] = -INFINITY;
        l_run[g] = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[g][j] = 0.f;
    }

    for (int i = 0; i < nt; ++i) {
        const int base = tile0 + i * kAttnWarps * WT;
        issue(i + kAttnStages - 1, end);
        cp_async_wait<kAttnStages - 1>();
        uint4 kr[UNR], vr[UNR];
        {
            const uint4* st = ring + (size_t)(i % kAttnStages) * UNR * 2 * 32;
#pragma unroll
            for (int u = 0; u < UNR; ++u) {
                kr[u] = st[(u * 2 + 0) * 32 + lane];
                vr[u] = st[(u * 2 + 1) * 32 + lane];
            }
        }
        if (p.early_kv && i < kAttnStages - 1) {
#pragma unroll
            for (int u = 0; u < UNR; ++u) {
                const int pos = base + u * PPW + pidx;
                if (cact && pos == L - 1 && pos < end) {
                    kr[u] = ldg16(kb + (int64_t)pos * p.ss);
                    vr[u] = ldg16(vb + (int64_t)pos * p.ss);
                }
            }
        }
        float s[UNR][G];
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
                s[u][g] = (base + u * PPW + pidx < end) ? d : -INFINITY;
            }
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float mt = s[0][g];
#pragma unroll
            for (int u = 1; u < UNR; ++u) mt = fmaxf(mt, s[u][g]);
#pragma unroll
            for (int o = LP; o < 32; o <<= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
            const float m_new = fmaxf(m_run[g], mt);
            const float alpha = exp2f(m_run[g] - m_new);
            l_run[g] *= alpha;
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[g][j] *= alpha;
#pragma unroll
            for (int u = 0; u < UNR; ++u) {
                const float pr = exp2f(s[u][g] - m_new);
                l_run[g] += pr;
                float vf[8];
                unpack8(vr[u], vf);
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[g][j] = fmaf(pr, vf[j], acc[g][j]);
            }
            m_run[g] = m_new;
        }
    }

    cp_async_wait<0>();

    // merge the PPW position groups of the warp (same running max: it is warp-uniform)
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int o = LP; o < 32; o <<= 1) {
            l_run[g] += __shfl_xor_sync(0xffffffffu, l_run[g], o);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[g][j] += __shfl_xor_sync(0xffffffffu, acc[g][j], o);
        }
    }
    if (pidx == 0 && cact) {
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
    __syncthreads();

    const bool direct = n_used <= 1;
    for (int idx = threadIdx.x; idx < nh * D; idx += kAttnThreads) {
        const int g = idx / D, d = idx - (idx / D) * D;
        float M = s_m[0][g];
#pragma unroll
        for (int w = 1; w < kAttnWarps; ++w) M = fmaxf(M, s_m[w][g]);
        float Ls = 0.f, A = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kAttnWarps; ++w) {
                const float sc = exp2f(s_m[w][g] - M);
                Ls = fmaf(s_l[w][g], sc, Ls);
                A = fmaf(s_acc[w][g][d], sc, A);
            }
        }
        const int h = h0 + g;
        if (direct) {
            p.out[(int64_t)b * p.o_sb + (int64_t)h * D + d] = __float2half_rn(Ls > 0.f ? A / Ls : 0.f);
        } else {
            const int64_t r = ((int64_t)b * p.nq + h) * p.splits + split;
            p.part[r * D + d] = A;
            if (d == 0) p.ml[r] = make_float2(M, Ls);
        }
    }
    if (direct) {
        __syncthreads();
        trace_end(p.trace);
        return;
    }

    // ---- last CTA of this (sequence, kv head, head group) merges the splits
    __shared__ int s_last;
    __threadfence();
    __syncthreads();
    int* ctr = p.counters + ((int64_t)b * p.nkv + kvh) * p.hg + hgi;
    if (threadIdx.x == 0) s_last = atomicAdd(ctr, 1) == n_used - 1;
    __syncthreads();
    if (!s_last) {
        trace_end(p.trace);
        return;
    }
    __threadfence();
    // per head: normalised weight of every split, exp2(m_s - M) / sum, in shared memory
    for (int g = warp; g < nh; g += kAttnWarps) {
        const int64_t r0 = ((int64_t)b * p.nq + h0 + g) * p.splits;
        float2 t[kMaxSplits / 32];
        float M = -INFINITY;
#pragma unroll
        for (int i = 0; i < kMaxSplits / 32; ++i) {
            const int sp = lane + 32 * i;
            t[i] = sp < n_used ? __ldcg(&p.ml[r0 + sp]) : make_float2(-INFINITY, 0.f);
            M = fmaxf(M, t[i].x);
        }
        M = warp_max(M);
        float Ls = 0.f;
#pragma unroll
        for (int i = 0; i < kMaxSplits / 32; ++i) {
            t[i].x = t[i].x == -INFINITY ? 0.f : exp2f(t[i].x - M);
            Ls = fmaf(t[i].y, t[i].x, Ls);
        }
        Ls = warp_sum(Ls);
        const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
#pragma unroll
        for (int i = 0; i < kMaxSplits / 32; ++i) {
            const int sp = lane + 32 * i;
            if (sp < n_used) s_w[g][sp] = t[i].x * inv;
        }
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < nh * D; idx += kAttnThreads) {
        const int g = idx / D, d = idx - (idx / D) * D;
        const float* pp = p.part + ((int64_t)b * p.nq + h0 + g) * p.splits * D + d;
        float A = 0.f;
#pragma unroll 8
        for (int sp = 0; sp < n_used; ++sp) A = fmaf(__ldcg(pp + (int64_t)sp * D), s_w[g][sp], A);
        p.out[(int64_t)b * p.o_sb + (int64_t)(h0 + g) * D + d] = __float2half_rn(A);
    }
    if (threadIdx.x == 0) *ctr = 0;
    __syncthreads();
    trace_end(p.trace);
}

template <int G>
constexpr size_t attn_ring_bytes() {
    return (size_t)kAttnWarps * kAttnStages * (G <= 4 ? 4 : 2) * 2 * 32 * sizeof(uint4);
}

template <int D, int G>
static cudaError_t launch_decode_dg(const AttnParams& p, dim3 grid, cudaStream_t s, bool pdl) {
    auto kern = attn_decode_kernel<D, G>;
    constexpr size_t smem = attn_ring_bytes<G>();
    static thread_local int set_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev != set_dev) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        set_dev = dev;
    }
    return launch(kern, grid, dim3(kAttnThreads), smem, s, pdl, p);
}

template <int D>
static cudaError_t launch_decode_d(const AttnParams& p, dim3 grid, int G, cudaStream_t s, bool pdl) {
    switch (G) {
        case 1: return launch_decode_dg<D, 1>(p, grid, s, pdl);
        case 2: return launch_decode_dg<D, 2>(p, grid, s, pdl);
        case 4: return launch_decode_dg<D, 4>(p, grid, s, pdl);
        default: return launch_decode_dg<D, 8>(p, grid, s, pdl);
    }
}

bool attn_head_dim_supported(int D) {
    return D == 16 || D == 32 || D == 48 || D == 64 || D == 96 || D == 128 || D == 256;
}

// Split count for `batch` sequences of at most max_len tokens given room for
// `cap_floats` of scratch (0: none).  Targets about four CTAs per SM.
int attn_head_groups(int nq, int nkv) {
    const int group = nq / nkv;
    const int G = group <= 1 ? 1 : (group <= 2 ? 2 : (group <= 4 ? 4 : 8));
    return (group + G - 1) / G;
}

// Scratch floats for `splits` > 1: partials, (max, sum) pairs, counters.
size_t attn_scratch_floats(int batch, int nq, int nkv, int D, int splits) {
    if (splits <= 1) return 0;
    return (size_t)batch * nq * splits * (D + 2) + (size_t)batch * nkv * attn_head_groups(nq, nkv);
}

int attn_pick_splits(int batch, int nq, int nkv, int D, int max_len, size_t cap_floats) {
    const long ctas1 = (long)batch * nkv * attn_head_groups(nq, nkv);
    const long target = 4L * sm_count();
    long splits = (target + ctas1 - 1) / ctas1;
    const long by_len = (max_len + 15) / 16;  // the kernel runs at least 16 positions per split
    if (splits > by_len) splits = by_len;
    if (splits > kMaxSplits) splits = kMaxSplits;
    while (splits > 1 && attn_scratch_floats(batch, nq, nkv, D, (int)splits) > cap_floats) --splits;
    if (splits < 1) splits = 1;
    return (int)splits;
}

// Launch the attention kernel.  When splits > 1, part must hold
// attn_scratch_floats() floats whose counter region is zero.
int attn_decode_launch(AttnParams p, int batch, int D, cudaStream_t s, bool pdl) {
    if (!attn_head_dim_supported(D)) return B2_ERR_UNSUPPORTED;
    const int group = p.nq / p.nkv;
    int G = group <= 1 ? 1 : (group <= 2 ? 2 : (group <= 4 ? 4 : 8));
    p.group = group;
    p.hg = (group + G - 1) / G;
    if (p.splits > 1) {
        p.ml = reinterpret_cast<float2*>(p.part + (size_t)batch * p.nq * p.splits * D);
        p.counters = reinterpret_cast<int*>(p.ml + (size_t)batch * p.nq * p.splits);
    }
    dim3 grid((unsigned)p.splits, (unsigned)(p.nkv * p.hg), (unsigned)batch);
    cudaError_t e;
    switch (D) {
        case 16: e = launch_decode_d<16>(p, grid, G, s, pdl); break;
        case 32: e = launch_decode_d<32>(p, grid, G, s, pdl); break;
        case 48: e = launch_decode_d<48>(p, grid, G, s, pdl); break;
        case 64: e = launch_decode_d<64>(p, grid, G, s, pdl); break;
        case 96: e = launch_decode_d<96>(p, grid, G, s, pdl); break;
        case 128: e = launch_decode_d<128>(p, grid, G, s, pdl); break;
        default: e = launch_decode_d<256>(p, grid, G, s, pdl); break;
    }
    if (e != cudaSuccess) return (int)e;
    return B2_OK;
}

static bool view_ok(const b2_kv_view& v) {
    return v.data && v.stride_d == 1 && aligned16(v.data) && (v.stride_b % 8 == 0) && (v.stride_h % 8 == 0) &&
           (v.stride_s % 8 == 0);
}

}  // namespace b2

namespace b2 {
}

using namespace b2;

extern "C" int b2_decode_gqa_split(const void* q, b2_kv_view kv, b2_kv_view vv, const int* seq_lens, void* out,
                                   int B, int nq, int nkv, int D, int max_seq_len, float* split_buffer,
                                   size_t split_buffer_floats, void* stream) {
    if (B <= 0) return B2_OK;
    B2_REQUIRE(q && out && seq_lens && nq > 0 && nkv > 0 && nq % nkv == 0 && max_seq_len >= 0);
    if (!attn_head_dim_supported(D)) return B2_ERR_UNSUPPORTED;
    if (!view_ok(kv) || !view_ok(vv) || kv.stride_b != vv.stride_b || kv.stride_h != vv.stride_h ||
        kv.stride_s != vv.stride_s || !aligned16(q) || !aligned16(out))
        return B2_ERR_UNSUPPORTED;
    {   // cluster-merged kernel: no scratch needed (split_buffer unused)
        const int rc = attn_cl_launch((const __half*)q, (int64_t)nq * D, (__half*)out, (int64_t)nq * D,
                                      (const __half*)kv.data, (const __half*)vv.data, kv.stride_b, kv.stride_h,
                                      kv.stride_s, max_seq_len, seq_lens, 0, B, nq, nkv, D, 0, 0, TraceSlot{nullptr, 0},
                                      as_stream(stream), true);
        if (rc != B2_ERR_UNSUPPORTED) return rc;
    }
    AttnParams p = {};
    p.q = (const __half*)q;
    p.q_sb = (int64_t)nq * D;
    p.k = (const __half*)kv.data;
    p.v = (const __half*)vv.data;
    p.sb = kv.stride_b;
    p.sh = kv.stride_h;
    p.ss = kv.stride_s;
    p.seq_lens = seq_lens;
    p.causal_base = -1;
    p.out = (__half*)out;
    p.o_sb = (int64_t)nq * D;
    p.nq = nq;
    p.nkv = nkv;
    p.scale_log2 = 1.4426950408889634f / sqrtf((float)D);
    p.part = split_buffer;
    p.splits = attn_pick_splits(B, nq, nkv, D, max_seq_len, split_buffer ? split_buffer_floats : 0);
    if (p.splits > 1) {
        // the caller's buffer holds arbitrary data: zero the arrival counters
        const size_t off = (size_t)B * nq * p.splits * (D + 2);
        const size_t n = attn_scratch_floats(B, nq, nkv, D, p.splits) - off;
        B2_TRY(cudaMemsetAsync(split_buffer + off, 0, n * sizeof(int), as_stream(stream)));
    }
    return attn_decode_launch(p, B, D, as_stream(stream), true);
}

extern "C" int b2_decode_gqa(const void* q, const void* kc, const void* vc, void* out, int total_seq_len, int nq,
                             int nkv, int max_seq, int D, void* stream) {
    if (total_seq_len <= 0) return B2_OK;
    B2_REQUIRE(q && kc && vc && out && nq > 0 && nkv > 0 && nq % nkv == 0 && total_seq_len <= max_seq);
    if (!attn_head_dim_supported(D) || !aligned16(q) || !aligned16(kc) || !aligned16(vc) || !aligned16(out))
        return B2_ERR_UNSUPPORTED;
    {
        const int rc = attn_cl_launch((const __half*)q, (int64_t)nq * D, (__half*)out, (int64_t)nq * D,
                                      (const __half*)kc, (const __half*)vc, 0, (int64_t)max_seq * D, D, max_seq,
                                      nullptr, total_seq_len, 1, nq, nkv, D, 0, 0, TraceSlot{nullptr, 0},
                                      as_stream(stream), true);
        if (rc != B2_ERR_UNSUPPORTED) return rc;
    }
    AttnParams p = {};
    p.q = (const __half*)q;
    p.q_sb = (int64_t)nq * D;
    p.k = (const __half*)kc;
    p.v = (const __half*)vc;
    p.sb = 0;
    p.sh = (int64_t)max_seq * D;
    p.ss = D;
    p.seq_lens = nullptr;
    p.len_const = total_seq_len;
    p.causal_base = -1;
    p.out = (__half*)out;
    p.o_sb = (int64_t)nq * D;
    p.nq = nq;
    p.nkv = nkv;
    p.scale_log2 = 1.4426950408889634f / sqrtf((float)D);
    p.splits = 1;
    return attn_decode_launch(p, 1, D, as_stream(stream), true);
}

namespace b2 {
// Causal attention through the decode kernel: query row i of batch element
// bb is a "sequence" of length i+1 over the token-major K/V of bb.  ldq,
// ldkv, ldo: elements between consecutive tokens (heads D apart in a row).
int causal_attention_rows_ld(const __half* q, int64_t ldq, const __half* k, const __half* v, int64_t ldkv,
                             __half* out, int64_t ldo, int64_t S, int nq, int nkv, int D, int batch,
                             cudaStream_t s) {
    for (int bb = 0; bb < batch; ++bb) {
        AttnParams p = {};
        p.q = q + (int64_t)bb * S * ldq;
        p.q_sb = ldq;
        p.k = k + (int64_t)bb * S * ldkv;
        p.v = v + (int64_t)bb * S * ldkv;
        p.sb = 0;
        p.sh = D;
        p.ss = ldkv;
        p.causal_base = 0;
        p.out = out + (int64_t)bb * S * ldo;
        p.o_sb = ldo;
        p.nq = nq;
        p.nkv = nkv;
        p.scale_log2 = 1.4426950408889634f / sqrtf((float)D);
        p.splits = 1;
        for (int64_t r0 = 0; r0 < S; r0 += 65535) {
            AttnParams pr = p;
            const int64_t rows = S - r0 < 65535 ? S - r0 : 65535;
            pr.q = p.q + r0 * p.q_sb;
            pr.out = p.out + r0 * p.o_sb;
            pr.causal_base = (int)r0;
            const int rc = attn_decode_launch(pr, (int)rows, D, s, true);
            if (rc != B2_OK) return rc;
        }
    }
    return B2_OK;
}

int causal_attention_rows(const __half* q, const __half* k, const __half* v, __half* out, int64_t S, int nq,
                          int nkv, int D, int batch, cudaStream_t s) {
    return causal_attention_rows_ld(q, (int64_t)nq * D, k, v, (int64_t)nkv * D, out, (int64_t)nq * D, S, nq, nkv, D,
                                    batch, s);
}
}  // namespace b2

extern "C" int b2_causal_gqa(const void* q, const void* k, const void* v, void* out, int64_t S, int64_t nq,
                             int64_t nkv, int64_t D, void* stream) {
    if (S <= 0) return B2_OK;
    B2_REQUIRE(q && k && v && out && nq > 0 && nkv > 0 && nq % nkv == 0);
    if (!attn_head_dim_supported((int)D) || !aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
        return B2_ERR_UNSUPPORTED;
    return causal_attention_rows((const __half*)q, (const __half*)k, (const __half*)v, (__half*)out, S, (int)nq,
                                 (int)nkv, (int)D, 1, as_stream(stream));
}

namespace b2 {
// Model-side launch: q/out [B][nq*D], K/V of one layer through (sb, sh, ss).
int attn_decode_launch_model(const __half* q, const __half* kbase, const __half* vbase, int64_t sb, int64_t sh,
                             int64_t ss, const int* seq_lens, __half* out, float* part, int splits, int B, int nq,
                             int nkv, int D, cudaStream_t s, bool pdl) {
    AttnParams p = {};
    p.q = q;
    p.q_sb = (int64_t)nq * D;
    p.k = kbase;
    p.v = vbase;
    p.sb = sb;
    p.sh = sh;
    p.ss = ss;
    p.seq_lens = seq_lens;
    p.causal_base = -1;
    p.out = out;
    p.o_sb = (int64_t)nq * D;
    p.nq = nq;
    p.nkv = nkv;
    p.scale_log2 = 1.4426950408889634f / sqrtf((float)D);
    p.part = part;
    p.splits = splits;
    return attn_decode_launch(p, B, D, s, pdl);
}

// Decode-step launch with q rows `q_sb` elements apart (the batched step
// reads q in place from the fused q|k|v rows).
int attn_decode_launch_step_q(const __half* q, int64_t q_sb, const __half* kbase, const __half* vbase, int64_t sb,
                              int64_t sh, int64_t ss, const int* seq_lens, __half* out, float* part, int splits,
                              int B, int nq, int nkv, int D, cudaStream_t s) {
    AttnParams p = {};
    p.q = q;
    p.q_sb = q_sb;
    p.k = kbase;
    p.v = vbase;
    p.sb = sb;
    p.sh = sh;
    p.ss = ss;
    p.seq_lens = seq_lens;
    p.causal_base = -1;
    p.out = out;
    p.o_sb = (int64_t)nq * D;
    p.nq = nq;
    p.nkv = nkv;
    p.scale_log2 = 1.4426950408889634f / sqrtf((float)D);
    p.part = part;
    p.splits = splits;
    p.early_kv = 1;
    return attn_decode_launch(p, B, D, s, true);
}

// Decode-step launch: as attn_decode_launch_model, and in addition the K/V
// rows older than seq_lens[b] - 1 and seq_lens itself are read before the
// programmatic-launch wait (valid only when the preceding kernel writes no
// more than the newest row).
int attn_decode_launch_step(const __half* q, const __half* kbase, const __half* vbase, int64_t sb, int64_t sh,
                            int64_t ss, const int* seq_lens, __half* out, float* part, int splits, int B, int nq,
                            int nkv, int D, cudaStream_t s, TraceSlot trace) {
    AttnParams p = {};
    p.q = q;
    p.q_sb = (int64_t)nq * D;
    p.k = kbase;
    p.v = vbase;
    p.sb = sb;
    p.sh = sh;
    p.ss = ss;
    p.seq_lens = seq_lens;
    p.causal_base = -1;
    p.out = out;
    p.o_sb = (int64_t)nq * D;
    p.nq = nq;
    p.nkv = nkv;
    p.scale_log2 = 1.4426950408889634f / sqrtf((float)D);
    p.part = part;
    p.splits = splits;
    p.early_kv = 1;
    p.trace = trace;
    return attn_decode_launch(p, B, D, s, true);
}
}  // namespace b2
