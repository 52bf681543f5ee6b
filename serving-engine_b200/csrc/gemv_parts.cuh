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

// Stage x for BT sequences into xs[BT][K8] (packed half).  Ends with a
// __syncthreads; every thread of the block must call it.
template <int BT, int XM, int NT>
__device__ __forceinline__ void stage_x(const GemvParams& p, uint4* __restrict__ xs, float* s_rs,
                                        float (*s_ss)[NT / 32], int lane, int warp) {
    const int K8 = p.K >> 3;
    if constexpr (XM == X_SUM) {
        // h = hid_in + every rank's tagged partial words, summed in rank
        // order; staged as half in xs, then normalised in place once the
        // CTA has the sum of squares.  Loads for two ranks at a time are
        // issued together (one L2 round trip per pair of ranks per chunk).
        const unsigned tag = (unsigned)(*p.tpx.step) * (unsigned)p.nslots + (unsigned)p.slot + 1u;
        const unsigned par = tag & 1u;
        float ss[BT];
#pragma unroll
        for (int b = 0; b < BT; ++b) ss[b] = 0.f;
        for (int i = threadIdx.x; i < BT * K8; i += NT) {
            const int b = i / K8, c = i - b * K8;
            uint4 o = make_uint4(0, 0, 0, 0);
            if (b < p.B) {
                float h[8];
                {
                    const float4* hr = reinterpret_cast<const float4*>(p.hid_in + (size_t)b * p.ldx) + 2 * c;
                    const float4 a0 = __ldcg(hr), a1 = __ldcg(hr + 1);
                    h[0] = a0.x; h[1] = a0.y; h[2] = a0.z; h[3] = a0.w;
                    h[4] = a1.x; h[5] = a1.y; h[6] = a1.z; h[7] = a1.w;
                }
                for (int r0 = 0; r0 < p.tpx.tp; r0 += 2) {
                    unsigned long long w[2][8];
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        if (r0 + q < p.tpx.tp) {
                            const unsigned long long* src =
                                p.tpx.recv + (((size_t)par * p.tpx.tp + r0 + q) * p.tpx.Bmax + b) * p.tpx.H + 8 * (size_t)c;
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
                        if (r0 + q < p.tpx.tp) {
                            const unsigned long long* src =
                                p.tpx.recv + (((size_t)par * p.tpx.tp + r0 + q) * p.tpx.Bmax + b) * p.tpx.H + 8 * (size_t)c;
#pragma unroll
                            for (int k = 0; k < 8; k += 2) {
                                float2 v;
                                if ((unsigned)(w[q][k] >> 32) == tag && (unsigned)(w[q][k + 1] >> 32) == tag)
                                    v = make_float2(__uint_as_float((unsigned)w[q][k]), __uint_as_float((unsigned)w[q][k + 1]));
                                else
                                    ll_load2(src + k, tag, v, p.tpx.err, 100 + p.slot);
                                h[k] += v.x;
                                h[k + 1] += v.y;
                            }
                        }
                    }
                }
                if (blockIdx.x == 0) {  // the residual stream after the exchange
                    float4* ho = reinterpret_cast<float4*>(p.hid_out + (size_t)b * p.ldx) + 2 * c;
                    ho[0] = make_float4(h[0], h[1], h[2], h[3]);
                    ho[1] = make_float4(h[4], h[5], h[6], h[7]);
                }
#pragma unroll
                for (int k = 0; k < 8; ++k) {
#pragma unroll
                    for (int bb = 0; bb < BT; ++bb)
                        if (bb == b) ss[bb] = fmaf(h[k], h[k], ss[bb]);
                }
                o = pack8(h);
            }
            xs[i] = o;
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
            if (b < p.B) {
                float f[8], wv[8];
                unpack8(xs[i], f);
                unpack8(ldg16(reinterpret_cast<const uint4*>(p.norm_w) + c), wv);
                const float r = s_rs[b];
#pragma unroll
                for (int k = 0; k < 8; ++k) f[k] = f[k] * r * wv[k];
                xs[i] = pack8(f);
            }
        }
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
                    __half* k = p.kcache + b * p.kv_sb + (int64_t)(h - p.nq) * p.kv_sh + (int64_t)pos * p.D;
                    k[i] = __float2half_rn(o1);
                    k[i + half] = __float2half_rn(o2);
                }
            } else {
                __half* v = p.vcache + b * p.kv_sb + (int64_t)(h - p.nq - p.nkv) * p.kv_sh + (int64_t)pos * p.D;
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
