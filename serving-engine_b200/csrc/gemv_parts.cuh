// gemv_parts.cuh -- the pieces every decode-GEMV kernel shares: staging of
// the activation vector in shared memory (plain half, RMSNorm of the fp32
// residual stream, or RMSNorm of the residual plus every tensor-parallel
// rank's partial), the per-task epilogues (bias / residual / RoPE + KV append
// / SwiGLU / logits + argmax / peer push), and the end-of-kernel work (peer
// push of a CTA's rows, argmax reduction and exchange).  Each is templated
// on the block's thread count NT.
#pragma once

#include <cmath>

#include "gemv.cuh"

namespace b2 {

__device__ __forceinline__ unsigned cluster_ctarank() {
    unsigned r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ unsigned cluster_nctarank() {
    unsigned r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_arrive_release() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Generic address of the same shared-memory object in cluster CTA `rank`.
template <typename T>
__device__ __forceinline__ const T* cluster_map(const T* p, unsigned rank) {
    uint64_t out;
    asm volatile("mapa.u64 %0, %1, %2;" : "=l"(out) : "l"(reinterpret_cast<uint64_t>(p)), "r"(rank));
    return reinterpret_cast<const T*>(out);
}

// Words of the exchange each lane reads per chunk of 8 elements: ranks 2g and
// 2g + 1 for lane g of the chunk's group of G2 lanes.
__device__ __forceinline__ int xsum_group_lanes(int tp) {
    const int g = (tp + 1) >> 1;
    return g <= 1 ? 1 : (g <= 2 ? 2 : 4);
}

// X_SUM staging, shared across the thread-block cluster.  The new residual
// h = hid_in + (sum of every rank's partial) is needed whole by every CTA
// (RMSNorm, then the GEMV's x), but each word of the exchange only has to
// cross L2 once per cluster: cluster CTA j sums chunks [j*per, (j+1)*per)
// of every sequence -- the G2 lanes of a chunk each load two ranks' tagged
// words, and a fixed butterfly combines them -- and keeps that slice of h
// (fp32) in its shared memory; after one cluster barrier every CTA reads the
// whole vector through distributed shared memory, normalises it and packs x.
// The sums use the same tree on every CTA of every rank, so all of them see
// bit-identical x; CTA 0 of the grid also stores h to hid_out (the residual
// stream after the exchange).  Every thread of the block calls it; the
// caller waits on the cluster barrier once more before exiting (a peer may
// still be reading this CTA's slice).
template <int BT, int NT>
__device__ __forceinline__ void stage_x_sum(const GemvParams& p, uint4* __restrict__ xs, float* s_rs,
                                            float (*s_ss)[NT / 32], int lane, int warp) {
    __shared__ float s_part[BT];
    const int K8 = p.K >> 3;
    const unsigned tag = (unsigned)(*p.tpx.step) * (unsigned)p.nslots + (unsigned)p.slot + 1u;
    const unsigned par = tag & 1u;
    const int tp = p.tpx.tp;
    const unsigned cs = cluster_nctarank(), cr = cluster_ctarank();
    const int per = (K8 + (int)cs - 1) / (int)cs;
    const int c0 = (int)cr * per;
    const int nown = max(0, min(K8, c0 + per) - c0);
    float* hsum = reinterpret_cast<float*>(xs + BT * K8);  // [BT][per][8] this CTA's slice of h
    const int G2 = xsum_group_lanes(tp);
    const int items = BT * nown * G2;
    float ss[BT];
#pragma unroll
    for (int b = 0; b < BT; ++b) ss[b] = 0.f;
    for (int base = 0; base < items; base += NT) {  // uniform trip count: the butterfly needs whole warps
        const int i = base + threadIdx.x;
        const bool act = i < items;
        int b = 0, cc = 0, g = 0;
        if (act) {
            g = i % G2;
            const int bc = i / G2;
            b = bc / nown;
            cc = bc - b * nown;
        }
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = 0.f;
        if (act && b < p.B) {
            const int c = c0 + cc;
            unsigned long long w[2][8];
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const int r = 2 * g + q;
                if (r < tp) {
                    const unsigned long long* src =
                        p.tpx.recv + (((size_t)par * tp + r) * p.tpx.Bmax + b) * p.tpx.H + 8 * (size_t)c;
#pragma unroll
                    for (int k = 0; k < 8; k += 2)
                        asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];"
                                     : "=l"(w[q][k]), "=l"(w[q][k + 1])
                                     : "l"(src + k)
                                     : "memory");
                }
            }
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const int r = 2 * g + q;
                if (r < tp) {
                    const unsigned long long* src =
                        p.tpx.recv + (((size_t)par * tp + r) * p.tpx.Bmax + b) * p.tpx.H + 8 * (size_t)c;
#pragma unroll
                    for (int k = 0; k < 8; k += 2) {
                        float2 x;
                        if ((unsigned)(w[q][k] >> 32) == tag && (unsigned)(w[q][k + 1] >> 32) == tag)
                            x = make_float2(__uint_as_float((unsigned)w[q][k]), __uint_as_float((unsigned)w[q][k + 1]));
                        else
                            ll_load2(src + k, tag, x, p.tpx.err, 100 + p.slot);
                        v[k] += x.x;
                        v[k + 1] += x.y;
                    }
                }
            }
        }
        for (int o = 1; o < G2; o <<= 1) {
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] += __shfl_xor_sync(0xffffffffu, v[k], o);
        }
        if (act && g == 0 && b < p.B) {
            const int c = c0 + cc;
            const float4* hr = reinterpret_cast<const float4*>(p.hid_in + (size_t)b * p.ldx) + 2 * c;
            const float4 a0 = __ldcg(hr), a1 = __ldcg(hr + 1);
            float h[8] = {a0.x + v[0], a0.y + v[1], a0.z + v[2], a0.w + v[3],
                          a1.x + v[4], a1.y + v[5], a1.z + v[6], a1.w + v[7]};
            float4* dst = reinterpret_cast<float4*>(hsum + ((size_t)b * per + cc) * 8);
            dst[0] = make_float4(h[0], h[1], h[2], h[3]);
            dst[1] = make_float4(h[4], h[5], h[6], h[7]);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
#pragma unroll
                for (int bb = 0; bb < BT; ++bb)
                    if (bb == b) ss[bb] = fmaf(h[k], h[k], ss[bb]);
            }
        }
    }
#pragma unroll
    for (int b = 0; b < BT; ++b) {
        const float v = warp_sum(ss[b]);
        if (lane == 0) s_ss[b][warp] = v;
    }
    __syncthreads();
    if (threadIdx.x < BT) {
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < (NT / 32); ++w) tot += s_ss[threadIdx.x][w];
        s_part[threadIdx.x] = tot;
    }
    cluster_arrive_release();
    cluster_wait_acquire();
    if (threadIdx.x < BT) {  // the whole vector's sum of squares, in cluster-rank order
        float tot = 0.f;
        for (unsigned j = 0; j < cs; ++j) tot += *cluster_map(&s_part[threadIdx.x], j);
        s_rs[threadIdx.x] = rsqrtf(tot / (float)p.K + p.eps);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < BT * K8; i += NT) {
        const int b = i / K8, c = i - b * K8;
        uint4 o = make_uint4(0, 0, 0, 0);
        if (b < p.B) {
            const int j = c / per, cc = c - j * per;
            const float4* src = cluster_map(reinterpret_cast<const float4*>(hsum + ((size_t)b * per + cc) * 8),
                                            (unsigned)j);
            const float4 a0 = src[0], a1 = src[1];
            if (blockIdx.x == 0) {  // the residual stream after the exchange
                float4* ho = reinterpret_cast<float4*>(p.hid_out + (size_t)b * p.ldx) + 2 * c;
                ho[0] = a0;
                ho[1] = a1;
            }
            float wv[8];
            unpack8(ldg16(reinterpret_cast<const uint4*>(p.norm_w) + c), wv);
            const float r = s_rs[b];
            float f[8] = {a0.x * r * wv[0], a0.y * r * wv[1], a0.z * r * wv[2], a0.w * r * wv[3],
                          a1.x * r * wv[4], a1.y * r * wv[5], a1.z * r * wv[6], a1.w * r * wv[7]};
            o = pack8(f);
        }
        xs[i] = o;
    }
    cluster_arrive_release();  // done reading the peers' slices; waited on before the kernel exits
    __syncthreads();
}

// Stage x for BT sequences into xs[BT][K8] (packed half).  Ends with a
// __syncthreads; every thread of the block must call it.
template <int BT, int XM, int NT>
__device__ __forceinline__ void stage_x(const GemvParams& p, uint4* __restrict__ xs, float* s_rs,
                                        float (*s_ss)[NT / 32], int lane, int warp) {
    const int K8 = p.K >> 3;
    if constexpr (XM == X_SUM) {
        stage_x_sum<BT, NT>(p, xs, s_rs, s_ss, lane, warp);
        return;
    } else if constexpr (XM == X_NORM) {
        const float* hrow = static_cast<const float*>(p.x);
        // Sum of squares of each sequence's fp32 residual row, spread over the
        // whole CTA so the loads are independent (one L2 round trip, not K/128).
        float ss[BT];
#pragma unroll
        for (int b = 0; b < BT; ++b) ss[b] = 0.f;
#pragma unroll 4
        for (int i = threadIdx.x; i < (p.K >> 2); i += NT) {
#pragma unroll
            for (int b = 0; b < BT; ++b) {
                if (b < p.B) {
                    const float4 v = reinterpret_cast<const float4*>(hrow + (size_t)b * p.ldx)[i];
                    ss[b] = fmaf(v.x, v.x, ss[b]); ss[b] = fmaf(v.y, v.y, ss[b]);
                    ss[b] = fmaf(v.z, v.z, ss[b]); ss[b] = fmaf(v.w, v.w, ss[b]);
                }
            }
        }
#pragma unroll
        for (int b = 0; b < BT; ++b) {
            const float v = warp_sum(ss[b]);
            if (lane == 0) s_ss[b][warp] = v;
        }
        __syncthreads();
        if (threadIdx.x < BT) {
            float tot = 0.f;
#pragma unroll
            for (int w = 0; w < (NT / 32); ++w) tot += s_ss[threadIdx.x][w];
            s_rs[threadIdx.x] = rsqrtf(tot / (float)p.K + p.eps);
        }
        __syncthreads();
        for (int i = threadIdx.x; i < BT * K8; i += NT) {
            const int b = i / K8, c = i - b * K8;
            uint4 o = make_uint4(0, 0, 0, 0);
            if (b < p.B) {
                const float4* hr = reinterpret_cast<const float4*>(hrow + (size_t)b * p.ldx) + 2 * c;
                const float4 a0 = hr[0], a1 = hr[1];
                float wv[8];
                unpack8(ldg16(reinterpret_cast<const uint4*>(p.norm_w) + c), wv);
                const float r = s_rs[b];
                float f[8] = {a0.x * r * wv[0], a0.y * r * wv[1], a0.z * r * wv[2], a0.w * r * wv[3],
                              a1.x * r * wv[4], a1.y * r * wv[5], a1.z * r * wv[6], a1.w * r * wv[7]};
                o = pack8(f);
            }
            xs[i] = o;
        }
    } else {
        const __half* xh = static_cast<const __half*>(p.x);
        for (int i = threadIdx.x; i < BT * K8; i += NT) {
            const int b = i / K8, c = i - b * K8;
            xs[i] = b < p.B ? ldg16(reinterpret_cast<const uint4*>(xh + (size_t)b * p.ldx) + c)
                            : make_uint4(0, 0, 0, 0);
        }
    }
    __syncthreads();

}

// Epilogue of task t once acc holds its warp-reduced dot products (every
// lane holds the sums); lane b handles sequence b.
template <int R, int BT, int OM>
__device__ __forceinline__ void task_epilogue(const GemvParams& p, int t, const float (&acc)[R][BT], int lane,
                                              unsigned long long (&best)[BT], float* s_push, int row0) {
    if constexpr (OM == OUT_LOGITS) {
#pragma unroll
        for (int b = 0; b < BT; ++b) {
            if (b < p.B) {
                const int gid = p.row_offset + t;
                if (gid < p.argmax_limit) {
                    const unsigned long long k = argmax_key(acc[0][b], (uint32_t)gid);
                    best[b] = k > best[b] ? k : best[b];
                }
            }
        }
    }
#pragma unroll
    for (int b = 0; b < BT; ++b) {
        if (lane != b || b >= p.B) continue;
        if constexpr (OM == OUT_HALF || OM == OUT_F32) {
            float v = acc[0][b];
            if (p.bias) v += __half2float(p.bias[t]);
            if (p.resid) v += __half2float(p.resid[(size_t)b * p.ld_resid + t]);
            if constexpr (OM == OUT_HALF)
                static_cast<__half*>(p.y)[(size_t)b * p.ldy + t] = __float2half_rn(v);
            else
                static_cast<float*>(p.y)[(size_t)b * p.ldy + t] = v;
        } else if constexpr (OM == OUT_RESID) {
            float* y = static_cast<float*>(p.y) + (size_t)b * p.ldy + t;
            *y = p.resid_add ? *y + acc[0][b] : acc[0][b];
        } else if constexpr (OM == OUT_PUSH) {
            s_push[b * kPushRows + (t - row0)] = acc[0][b];
        } else if constexpr (OM == OUT_LOGITS) {
            static_cast<float*>(p.y)[(size_t)b * p.ldy + t] = acc[0][b];
        } else if constexpr (OM == OUT_SWIGLU) {
            const float g = acc[0][b], u = acc[1][b];
            static_cast<__half*>(p.y)[(size_t)b * p.ldy + t] = __float2half_rn(g / (1.0f + expf(-g)) * u);
        } else if constexpr (OM == OUT_QKV) {
            const int half = p.D >> 1;
            const int h = t / half, i = t - h * half;
            float x1 = acc[0][b], x2 = acc[1][b];
            if (p.bias) {
                x1 += __half2float(p.bias[h * p.D + i]);
                x2 += __half2float(p.bias[h * p.D + i + half]);
            }
            const int pos = p.pos[b];
            if (h < p.nq + p.nkv) {
                const float2 cs = p.rope[(size_t)pos * half + i];
                const float o1 = x1 * cs.x - x2 * cs.y;
                const float o2 = x2 * cs.x + x1 * cs.y;
                if (h < p.nq) {
                    __half* q = static_cast<__half*>(p.y) + (size_t)b * p.ldy + h * p.D;
                    q[i] = __float2half_rn(o1);
                    q[i + half] = __float2half_rn(o2);
                } else {
                    __half* k = p.kv.k + kv_row(p.kv, b, h - p.nq, pos, p.D);
                    k[i] = __float2half_rn(o1);
                    k[i + half] = __float2half_rn(o2);
                }
            } else {
                __half* v = p.kv.v + kv_row(p.kv, b, h - p.nq - p.nkv, pos, p.D);
                v[i] = __float2half_rn(x1);
                v[i + half] = __float2half_rn(x2);
            }
        }
    }
}

// End-of-kernel work after every warp's tasks: OUT_PUSH sends the CTA's
// staged rows to every rank; OUT_LOGITS reduces the per-warp argmax keys
// (and, with the exchange on, hands the shard's argmax to every rank).
template <int BT, int OM, int NT>
__device__ __forceinline__ void gemv_finish(const GemvParams& p, int lane, int warp,
                                            const unsigned long long (&best)[BT],
                                            unsigned long long (*s_best)[BT], const float* s_push, int row0,
                                            int t_end, unsigned push_epoch, unsigned push_par) {
    if constexpr (OM == OUT_PUSH) {
        // this CTA's block of partial rows, as tagged 8-byte words (two per
        // 16-byte store) into slot [parity][rank] of every rank
        __syncthreads();
        const int n2 = (t_end - row0) >> 1;  // rows_per_cta and H are even
        const int per_rank = p.B * n2;
        for (int i = threadIdx.x; i < p.tpx.tp * per_rank; i += NT) {
            const int r = i / per_rank, rem = i - r * per_rank;
            const int b = rem / n2, c2 = rem - b * n2;
            unsigned long long* dst = p.tpx.peer_recv[r] +
                                      (((size_t)push_par * p.tpx.tp + p.tpx.rank) * p.tpx.Bmax + b) * p.tpx.H + row0 +
                                      2 * c2;
            ll_store2(dst, ll_word(s_push[b * kPushRows + 2 * c2], push_epoch), ll_word(s_push[b * kPushRows + 2 * c2 + 1], push_epoch));
        }
    }

    if constexpr (OM == OUT_LOGITS) {
        if (lane == 0) {
#pragma unroll
            for (int b = 0; b < BT; ++b) s_best[warp][b] = best[b];
        }
        __syncthreads();
        if (threadIdx.x < BT && (int)threadIdx.x < p.B) {
            unsigned long long m = 0ull;
            for (int w = 0; w < (NT / 32); ++w) m = s_best[w][threadIdx.x] > m ? s_best[w][threadIdx.x] : m;
            if (m) atomicMax(p.argmax + threadIdx.x, m);
        }
        if (p.tp_on) {
            // the last CTA hands this vocabulary shard's argmax to every rank
            __syncthreads();
            if (threadIdx.x == 0) {
                __threadfence();
                if (atomicAdd(p.tpx.ctr, 1) == (int)gridDim.x - 1) {
                    __threadfence();
                    const unsigned tag = (unsigned)(*p.tpx.step) + 1u;
                    for (int b = 0; b < p.B; ++b) {
                        const unsigned long long v = atomicAdd(p.argmax + b, 0ull);
                        for (int r = 0; r < p.tpx.tp; ++r)
                            p.tpx.peer_am_recv[r][(size_t)p.tpx.rank * p.tpx.Bmax + b] = v;
                    }
                    *p.tpx.ctr = 0;
                    fence_acq_rel_sys();
                    for (int r = 0; r < p.tpx.tp; ++r) store_release_sys(p.tpx.peer_am_flags[r] + p.tpx.rank, tag);
                }
            }
        }
    }
}

}  // namespace b2
