// prefill.cu -- causal GQA flash prefill on the tcgen05 tensor cores
// (operator API flash_prefill_gqa, plus a bf16 / fused-RoPE form).
//
// One CTA computes the attention output of one 128-query tile of one query
// head.  Q, K and V tiles (128 rows x D, 128-byte swizzled) arrive by TMA;
// both products run on the tensor cores with fp32 accumulation in TMEM:
//   S_j = Q K_j^T    M=128 queries, N=128 keys, K=D   (TMEM columns 0-255,
//                    two buffers, so S_{j+1} is computed while row j's
//                    softmax runs)
//   O  += P_j V_j    M=128 queries, N=D, K=128 keys  (TMEM columns 256..;
//                    columns 384.. hold the RoPE warps' angle tables)
// Warp roles (192 threads):
//   warp 4      TMA producer: Q once, then K_j / V_j into 2-stage rings;
//   warp 5      MMA issuer (one thread): S_j, then P_{j-1} V_{j-1};
//   warps 0..3  softmax, one query row per thread: per key tile the row
//               of S_j read from TMEM once into registers, causal mask, row
//               max, P_j = exp2(S scale - m) as half/bf16 into one of two
//               swizzled shared-memory P buffers (P_j is written while
//               P_{j-1} V_{j-1} runs), running row sum; O / l at the end.
// RoPE form: queries and keys are rotated once by a pre-pass kernel of the
// same call into dense copies that the Q and K tiles are loaded from.
// Online softmax without a rescale per tile: the reference max m of a row
// only moves when the tile max exceeds it by more than 8 (log2 units); P
// values stay <= 2^8 otherwise, and when m moves the O row in TMEM is scaled
// by exp2(m_old - m_new) before the next P V accumulates into it.
// Causal: tile qt needs KV tiles 0..qt; the diagonal tile is masked, tiles
// are scheduled heaviest first.  Every mbarrier wait is bounded (tc.cuh).
//
// Shapes the tensor-core kernel does not take (head_dim other than 64/128,
// unaligned bases) run each query row as a decode query of length i+1
// through the split-KV attention kernel (attention.cu).
// Reference replaced: src/cuda/flash_prefill.cu:43-240 (16 threads per CTA,
// one query row per thread, scalar FMA, head_dim fixed at 64).
#include <cmath>
#include <mutex>
#include <new>
#include <type_traits>

#include "prefill.cuh"
#include "tc.cuh"

namespace b2 {
int causal_attention_rows(const __half* q, const __half* k, const __half* v, __half* out, int64_t S, int nq,
                          int nkv, int D, int batch, cudaStream_t s);
bool attn_head_dim_supported(int D);

template <int D>
struct FlashCfg {
    static constexpr int ATOMS = D / 64;                    // 128-byte swizzle atoms per row
    static constexpr uint32_t ATOM = 128 * 128;             // bytes of one 128-row atom
    static constexpr uint32_t TILE = 128 * D * 2;           // Q, K or V tile
    static constexpr uint32_t P_BYTES = 128 * 128 * 2;
    static constexpr uint32_t OFF_Q = 0;
    static constexpr uint32_t OFF_K = TILE;                 // 2 stages
    static constexpr uint32_t OFF_V = 3 * TILE;             // 2 stages
    static constexpr uint32_t OFF_P = 5 * TILE;             // 2 buffers
    static constexpr uint32_t OFF_BAR = OFF_P + 2 * P_BYTES;
    // 1 KB alignment slack; at least 120 KB so that one CTA (and its 512 TMEM
    // columns) owns an SM
    static constexpr size_t SMEM_NEED = OFF_BAR + 256 + 1024;
    static constexpr size_t SMEM = SMEM_NEED > 122880 ? SMEM_NEED : 122880;
    static constexpr int THREADS = 192;
    static constexpr uint32_t TMEM_COLS = 512;
};

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    if constexpr (BF16) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    } else {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
}

template <bool BF16>
__device__ __forceinline__ float2 unpack2(uint32_t v) {
    if constexpr (BF16) {
        __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&v);
        return __bfloat1622float2(h);
    } else {
        __half2 h = *reinterpret_cast<__half2*>(&v);
        return __half22float2(h);
    }
}

// Byte offset of element e of row `row` in a 128-byte-swizzled tile made of
// 128-row atoms of 64 elements.
__device__ __forceinline__ uint32_t sw128_off(int row, int e) {
    return (uint32_t)(e >> 6) * (128u * 128u) + (uint32_t)row * 128u + ((((uint32_t)(e & 63) >> 3) ^ (row & 7)) << 4) +
           ((uint32_t)(e & 7) << 1);
}

// Rotate-half RoPE of the reference (src/cpu/ops.cpp:174-189): x[i],
// x[i+D/2] -> x[i] c - x[i+D/2] s, x[i+D/2] c + x[i] s with
// (c, s) = (cos, sin)(float(pos) * inv_freq[i]), inv_freq[i] =
// 1 / theta^(2i/D) -- the same float product per element as the reference.
//
// Queries and keys are rotated once, by a pre-pass of the same call, into
// dense [batch][S][heads][D] copies that the attention kernel's Q and K tiles
// are loaded from: rotating inside the attention CTAs would put the rotation
// on each CTA's path to its first S = Q K^T and repeat the keys' rotation
// S/128 * nq/nkv times.  One thread per (token, 8 frequencies, group of 8
// heads of the q|k head list): its 8 (cos, sin) pairs are computed once and
// applied to each head of the group.
template <bool BF16>
__global__ void rope_qk_kernel(const uint16_t* __restrict__ q, int64_t ldq, const uint16_t* __restrict__ k,
                               int64_t ldk, uint16_t* __restrict__ qo, uint16_t* __restrict__ ko, int S, int nq,
                               int nkv, int D, int batch, float theta, int pos0) {
    constexpr int kHeads = 8;
    __shared__ float invf[64];
    const int H = D / 2;
    if ((int)threadIdx.x < H) invf[threadIdx.x] = 1.0f / powf(theta, (float)(2 * threadIdx.x) / (float)D);
    __syncthreads();
    griddep_wait();
    const int chunks = H / 8;
    const int groups = (nq + nkv + kHeads - 1) / kHeads;
    const int64_t n = (int64_t)batch * S * groups * chunks;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % chunks) * 8;
        const int g = (int)((i / chunks) % groups);
        const int64_t bs = i / ((int64_t)chunks * groups);  // (b, s)
        const int pos = pos0 + (int)(bs % S);
        float cs[8], sn[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) sincosf((float)pos * invf[c + e], &sn[e], &cs[e]);
        const int h_end = min(nq + nkv, (g + 1) * kHeads);
#pragma unroll 4
        for (int hd = g * kHeads; hd < h_end; ++hd) {
            const bool isq = hd < nq;
            const uint16_t* src = isq ? q + bs * ldq + (int64_t)hd * D : k + bs * ldk + (int64_t)(hd - nq) * D;
            uint16_t* dst = isq ? qo + (bs * nq + hd) * D : ko + (bs * nkv + (hd - nq)) * D;
            uint4 a = *reinterpret_cast<const uint4*>(src + c), b = *reinterpret_cast<const uint4*>(src + c + H);
            uint32_t* aw = reinterpret_cast<uint32_t*>(&a);
            uint32_t* bw = reinterpret_cast<uint32_t*>(&b);
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                const float2 x1 = unpack2<BF16>(aw[w]), x2 = unpack2<BF16>(bw[w]);
                const float c0 = cs[2 * w], s0 = sn[2 * w], c1 = cs[2 * w + 1], s1 = sn[2 * w + 1];
                aw[w] = pack2<BF16>(x1.x * c0 - x2.x * s0, x1.y * c1 - x2.y * s1);
                bw[w] = pack2<BF16>(x2.x * c0 + x1.x * s0, x2.y * c1 + x1.y * s1);
            }
            *reinterpret_cast<uint4*>(dst + c) = a;
            *reinterpret_cast<uint4*>(dst + c + H) = b;
        }
    }
}

// 2^x on the SFU (ex2.approx, flush-to-zero): exp2(-inf) = 0, relative error
// ~2^-22, far below the half/bf16 rounding that P gets next.
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <int D, bool BF16>
__global__ void __launch_bounds__(FlashCfg<D>::THREADS, 1)
    flash_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, void* __restrict__ out, int64_t ldo, int S, int nq,
                    int nkv, float scale_log2, int* err) {
    using Cfg = FlashCfg<D>;
    constexpr uint32_t TILE = Cfg::TILE;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = sm + Cfg::OFF_Q;
    uint8_t* sK = sm + Cfg::OFF_K;
    uint8_t* sV = sm + Cfg::OFF_V;
    uint8_t* sP = sm + Cfg::OFF_P;
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm + Cfg::OFF_BAR);
    uint64_t* q_full = bar + 0;   // (bar + 1 spare)
    uint64_t* k_full = bar + 2;   // [2] (bar + 4, + 5 spare)
    uint64_t* k_empty = bar + 6;  // [2]
    uint64_t* v_full = bar + 8;   // [2]
    uint64_t* v_empty = bar + 10; // [2]
    uint64_t* s_full = bar + 12;  // [2]
    uint64_t* p_full = bar + 14;  // [2]
    uint64_t* o_done = bar + 16;  // [2]: P_j V_j done, committed on o_done[j & 1]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 18);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // grid (heads, tiles, batch): CTAs are dispatched x fastest, so every
    // head's heaviest tile goes out before any lighter one (longest first)
    const int qt = (int)gridDim.y - 1 - (int)blockIdx.y;
    const int h = blockIdx.x, b = blockIdx.z;
    const int kvh = h / (nq / nkv);
    const int q0 = qt * 128;
    const int nt = qt + 1;

    if (threadIdx.x == 0) {
        tc::mbar_init(q_full, 1);
        for (int s = 0; s < 2; ++s) {
            tc::mbar_init(&k_full[s], 1);
            tc::mbar_init(&k_empty[s], 1);
            tc::mbar_init(&v_full[s], 1);
            tc::mbar_init(&v_empty[s], 1);
            tc::mbar_init(&s_full[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            tc::mbar_init(&p_full[s], 128);
            tc::mbar_init(&o_done[s], 1);
        }
        tc::fence_barrier_init();
    }
    if (warp == 0) tc::tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tO = tmem + 256;

    griddep_wait();  // Q / K / V may be the previous kernel's output
    griddep_launch_dependents();

    if (warp == 4) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            tc::mbar_arrive_expect_tx(q_full, TILE);
#pragma unroll
            for (int a = 0; a < Cfg::ATOMS; ++a) tc::tma_load_4d(sQ + a * Cfg::ATOM, &tmQ, q_full, a * 64, h, q0, b);
            for (int j = 0; j < nt; ++j) {
                const int s = j & 1;
                const uint32_t u = (uint32_t)j >> 1;
                if (j >= 2 && !tc::mbar_wait(&k_empty[s], (u - 1) & 1u, err, 11)) break;
                tc::mbar_arrive_expect_tx(&k_full[s], TILE);
#pragma unroll
                for (int a = 0; a < Cfg::ATOMS; ++a)
                    tc::tma_load_4d(sK + s * TILE + a * Cfg::ATOM, &tmK, &k_full[s], a * 64, kvh, j * 128, b);
                if (j >= 2 && !tc::mbar_wait(&v_empty[s], (u - 1) & 1u, err, 12)) break;
                tc::mbar_arrive_expect_tx(&v_full[s], TILE);
#pragma unroll
                for (int a = 0; a < Cfg::ATOMS; ++a)
                    tc::tma_load_4d(sV + s * TILE + a * Cfg::ATOM, &tmV, &v_full[s], a * 64, kvh, j * 128, b);
            }
        }
    } else if (warp == 5) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idS = tc::idesc_f16(128, 128, BF16, false);
            constexpr uint32_t idO = tc::idesc_f16(128, D, BF16, true);
            const uint32_t aQ = tc::smem_u32(sQ), aK = tc::smem_u32(sK), aV = tc::smem_u32(sV),
                           aP = tc::smem_u32(sP);
            bool ok = tc::mbar_wait(q_full, 0, err, 13);
            for (int j = 0; ok && j <= nt; ++j) {
                if (j < nt) {
                    const int s = j & 1;
                    const uint32_t u = (uint32_t)j >> 1;
                    ok = tc::mbar_wait(&k_full[s], u & 1u, err, 14);
                    if (!ok) break;
                    tc::fence_after_sync();
#pragma unroll
                    for (int kk = 0; kk < D / 16; ++kk) {
                        const uint32_t off = (uint32_t)(kk >> 2) * Cfg::ATOM + (uint32_t)(kk & 3) * 32;
                        tc::mma_f16(tmem + s * 128, tc::desc_k_sw128(aQ + off), tc::desc_k_sw128(aK + s * TILE + off),
                                    idS, kk > 0 ? 1u : 0u);
                    }
                    tc::mma_commit(&s_full[s]);
                    tc::mma_commit(&k_empty[s]);
                }
                if (j > 0) {
                    const int jj = j - 1, s = jj & 1;
                    const uint32_t u = (uint32_t)jj >> 1;
                    ok = tc::mbar_wait(&p_full[s], u & 1u, err, 15) && tc::mbar_wait(&v_full[s], u & 1u, err, 16);
                    if (!ok) break;
                    tc::fence_after_sync();
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint32_t offp = (uint32_t)(kk >> 2) * Cfg::ATOM + (uint32_t)(kk & 3) * 32;
                        tc::mma_f16(tO, tc::desc_k_sw128(aP + s * Cfg::P_BYTES + offp),
                                    tc::desc_mn_sw128(aV + s * TILE + (uint32_t)kk * 2048u, Cfg::ATOM), idO,
                                    (jj > 0 || kk > 0) ? 1u : 0u);
                    }
                    tc::mma_commit(&o_done[s]);
                    tc::mma_commit(&v_empty[s]);
                }
            }
        }
    } else if (warp < 4) {
        // ---------------- softmax and output ----------------
        // Thread r owns query row r: S_j's row comes out of TMEM once (128
        // registers), is masked and reduced, and P_j = exp2(S scale - m) goes
        // to P buffer j & 1, so P_j is written while P_{j-1} V_{j-1} runs.
        // The O row is touched only when m moves (after P_{j-1} V_{j-1}).
        const int r = warp * 32 + lane;
        const int qpos = q0 + r;
        const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
        float m = -1e30f, l = 0.f;  // finite start: a fully masked row keeps P = 0 and l = 0
        bool ok = true;
        for (int j = 0; ok && j < nt; ++j) {
            const int s = j & 1;
            const uint32_t u = (uint32_t)j >> 1;
            ok = __all_sync(0xffffffffu, tc::mbar_wait(&s_full[s], u & 1u, err, 19));
            if (!ok) break;
            tc::fence_after_sync();
            uint32_t v[128];
            const uint32_t srow = tmem + lane_base + s * 128;
#pragma unroll
            for (int c = 0; c < 4; ++c)
                tc::tmem_ld32(srow + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&v[32 * c]));
            tc::tmem_wait_ld();
            const int kbase = j * 128;
            if (kbase + 127 > q0 || kbase + 128 > S) {  // diagonal or ragged tile (warp-uniform)
#pragma unroll
                for (int e = 0; e < 128; ++e)
                    if (kbase + e > qpos || kbase + e >= S) v[e] = 0xff800000u;  // -inf
            }
            float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int e = 0; e < 128; ++e) mx4[e & 3] = fmaxf(mx4[e & 3], __uint_as_float(v[e]));
            const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * scale_log2;
            const float m_new = fmaxf(m, mx);
            const bool resc = m_new > m + 8.f;
            const float m_use = resc ? m_new : m;
            const float alpha = fast_exp2(m - m_use);
            if (j > 0 && __any_sync(0xffffffffu, resc)) {
                // O must hold P_{j-1} V_{j-1} before this warp's rows are scaled
                const uint32_t jj = (uint32_t)(j - 1);
                ok = __all_sync(0xffffffffu, tc::mbar_wait(&o_done[jj & 1u], (jj >> 1) & 1u, err, 20));
                if (!ok) break;
                tc::fence_after_sync();
#pragma unroll 1
                for (int c = 0; c < D; c += 32) {
                    uint32_t o[32];
                    tc::tmem_ld32(tO + lane_base + c, o);
                    tc::tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
                    tc::tmem_st32(tO + lane_base + c, o);
                }
                tc::tmem_wait_st();
            }
            m = m_use;
            // P buffer s is free once P_{j-2} V_{j-2} has completed
            if (j >= 2) {
                ok = __all_sync(0xffffffffu, tc::mbar_wait(&o_done[s], (u - 1) & 1u, err, 22));
                if (!ok) break;
            }
            uint8_t* pbuf = sP + s * Cfg::P_BYTES;
            float l4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int c = 0; c < 128; c += 8) {
                uint32_t pk[4];
#pragma unroll
                for (int e = 0; e < 8; e += 2) {
                    const float p0 = fast_exp2(fmaf(__uint_as_float(v[c + e]), scale_log2, -m));
                    const float p1 = fast_exp2(fmaf(__uint_as_float(v[c + e + 1]), scale_log2, -m));
                    l4[e >> 1] += p0 + p1;
                    pk[e >> 1] = pack2<BF16>(p0, p1);
                }
                *reinterpret_cast<uint4*>(pbuf + sw128_off(r, c)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            }
            l = l * alpha + ((l4[0] + l4[1]) + (l4[2] + l4[3]));
            tc::fence_proxy_async_smem();
            tc::fence_before_sync();
            tc::mbar_arrive(&p_full[s]);
        }
        if (ok) {
            const uint32_t jl = (uint32_t)(nt - 1);
            ok = __all_sync(0xffffffffu, tc::mbar_wait(&o_done[jl & 1u], (jl >> 1) & 1u, err, 21));
        }
        tc::fence_after_sync();
        const float inv_l = l > 0.f ? 1.f / l : 0.f;
        using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
        T* orow = static_cast<T*>(out) + ((int64_t)b * S + qpos) * ldo + (int64_t)h * D;
#pragma unroll 1
        for (int c = 0; c < D; c += 32) {
            uint32_t v[32];
            tc::tmem_ld32(tO + lane_base + c, v);
            tc::tmem_wait_ld();
            if (!ok || qpos >= S) continue;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                uint4 w;
                w.x = pack2<BF16>(__uint_as_float(v[8 * q + 0]) * inv_l, __uint_as_float(v[8 * q + 1]) * inv_l);
                w.y = pack2<BF16>(__uint_as_float(v[8 * q + 2]) * inv_l, __uint_as_float(v[8 * q + 3]) * inv_l);
                w.z = pack2<BF16>(__uint_as_float(v[8 * q + 4]) * inv_l, __uint_as_float(v[8 * q + 5]) * inv_l);
                w.w = pack2<BF16>(__uint_as_float(v[8 * q + 6]) * inv_l, __uint_as_float(v[8 * q + 7]) * inv_l);
                *reinterpret_cast<uint4*>(orow + c + 8 * q) = w;
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, Cfg::TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------
// Two-Q-tile form (head_dim 128): one CTA computes two consecutive 128-query
// tiles A and B of one head, so the tensor core always has the other tile's
// work while one tile's softmax runs, and P stays in TMEM.
//   TMEM (512 columns): tile t's S_j / P_j at 256 t (P_j, 16-bit, packed two
//   per column, overwrites the first 64 columns of S_j once the softmax has
//   read S_j), its O at 256 t + 128.
//   MMA order per key tile j: PV_A,j, S_A,j+1, PV_B,j, S_B,j+1 -- each S is
//   issued behind the PV that reads the P it overwrites, and its completion
//   (s_full) also tells the softmax that the previous PV is done, so the O
//   rescale and the P write need no other wait.
//   PV_t,j = P_t,j (A operand read from TMEM) x V_j (MN-major, shared memory).
// Warps: 0..3 softmax of tile A, 4..7 of tile B (one query row per thread),
// 8 TMA producer (Q_A, Q_B once, K/V 2-stage rings shared by both tiles),
// 9 MMA issuer.  Causal: tile A needs key tiles 0..2p, tile B 0..2p+1.
// ---------------------------------------------------------------------------
struct F2Cfg {
    static constexpr uint32_t TILE = 128 * 128 * 2;  // a Q, K or V tile (D = 128)
    static constexpr uint32_t ATOM = 128 * 128;
    static constexpr uint32_t OFF_Q = 0;             // 2 tiles
    static constexpr uint32_t OFF_K = 2 * TILE;      // 2 stages
    static constexpr uint32_t OFF_V = 4 * TILE;      // 2 stages
    static constexpr uint32_t OFF_BAR = 6 * TILE;
    static constexpr size_t SMEM = OFF_BAR + 256 + 1024;
    static constexpr int THREADS = 320;
};

template <bool BF16>
__global__ void __launch_bounds__(F2Cfg::THREADS, 1)
    flash2_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, void* __restrict__ out, int64_t ldo, int S, int nq,
                     int nkv, float scale_log2, int* err) {
    constexpr int D = 128;
    constexpr uint32_t TILE = F2Cfg::TILE, ATOM = F2Cfg::ATOM;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = sm + F2Cfg::OFF_Q;
    uint8_t* sK = sm + F2Cfg::OFF_K;
    uint8_t* sV = sm + F2Cfg::OFF_V;
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm + F2Cfg::OFF_BAR);
    uint64_t* q_full = bar + 0;    // (bar + 1 spare)
    uint64_t* k_full = bar + 2;    // [2]
    uint64_t* k_empty = bar + 4;   // [2]
    uint64_t* v_full = bar + 6;    // [2]
    uint64_t* v_empty = bar + 8;   // [2]
    uint64_t* s_full = bar + 10;   // [tile]
    uint64_t* p_full = bar + 12;   // [tile]
    uint64_t* o_done = bar + 14;   // [tile]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 16);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // grid (heads, pairs, batch): every head's heaviest pair is dispatched
    // before any lighter one (longest first across the whole grid)
    const int pt = (int)gridDim.y - 1 - (int)blockIdx.y;
    const int h = blockIdx.x, b = blockIdx.z;
    const int kvh = h / (nq / nkv);
    const int q0 = pt * 256;
    const bool hasB = q0 + 128 < S;
    const int ntA = 2 * pt + 1;
    const int ntB = hasB ? 2 * pt + 2 : 0;
    const int nt = hasB ? ntB : ntA;

    if (threadIdx.x == 0) {
        tc::mbar_init(q_full, 1);
        for (int s = 0; s < 2; ++s) {
            tc::mbar_init(&k_full[s], 1);
            tc::mbar_init(&k_empty[s], 1);
            tc::mbar_init(&v_full[s], 1);
            tc::mbar_init(&v_empty[s], 1);
            tc::mbar_init(&s_full[s], 1);
            tc::mbar_init(&p_full[s], 128);
            tc::mbar_init(&o_done[s], 1);
        }
        tc::fence_barrier_init();
    }
    if (warp == 0) tc::tmem_alloc(tmem_slot, 512);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    griddep_wait();
    griddep_launch_dependents();

    if (warp == 8) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            tc::mbar_arrive_expect_tx(q_full, 2 * TILE);
#pragma unroll
            for (int t = 0; t < 2; ++t)
#pragma unroll
                for (int a = 0; a < 2; ++a)
                    tc::tma_load_4d(sQ + t * TILE + a * ATOM, &tmQ, q_full, a * 64, h, q0 + t * 128, b);
            for (int j = 0; j < nt; ++j) {
                const int s = j & 1;
                const uint32_t u = (uint32_t)j >> 1;
                if (j >= 2 && !tc::mbar_wait(&k_empty[s], (u - 1) & 1u, err, 31)) break;
                tc::mbar_arrive_expect_tx(&k_full[s], TILE);
#pragma unroll
                for (int a = 0; a < 2; ++a)
                    tc::tma_load_4d(sK + s * TILE + a * ATOM, &tmK, &k_full[s], a * 64, kvh, j * 128, b);
                if (j >= 2 && !tc::mbar_wait(&v_empty[s], (u - 1) & 1u, err, 32)) break;
                tc::mbar_arrive_expect_tx(&v_full[s], TILE);
#pragma unroll
                for (int a = 0; a < 2; ++a)
                    tc::tma_load_4d(sV + s * TILE + a * ATOM, &tmV, &v_full[s], a * 64, kvh, j * 128, b);
            }
        }
    } else if (warp == 9) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idS = tc::idesc_f16(128, 128, BF16, false);
            constexpr uint32_t idO = tc::idesc_f16(128, D, BF16, true);
            const uint32_t aQ = tc::smem_u32(sQ), aK = tc::smem_u32(sK), aV = tc::smem_u32(sV);
            auto issue_s = [&](int t, int j) {
                const uint32_t kb = aK + (uint32_t)(j & 1) * TILE, qb = aQ + (uint32_t)t * TILE;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t off = (uint32_t)(kk >> 2) * ATOM + (uint32_t)(kk & 3) * 32;
                    tc::mma_f16(tmem + (uint32_t)t * 256, tc::desc_k_sw128(qb + off), tc::desc_k_sw128(kb + off), idS,
                                kk > 0 ? 1u : 0u);
                }
                tc::mma_commit(&s_full[t]);
            };
            auto issue_pv = [&](int t, int j) {
                const uint32_t vb = aV + (uint32_t)(j & 1) * TILE;
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    tc::mma_f16_ts(tmem + (uint32_t)t * 256 + 128, tmem + (uint32_t)t * 256 + (uint32_t)kk * 8,
                                   tc::desc_mn_sw128(vb + (uint32_t)kk * 2048u, ATOM), idO, (j > 0 || kk > 0) ? 1u : 0u);
                tc::mma_commit(&o_done[t]);
            };
            bool ok = tc::mbar_wait(q_full, 0, err, 33) && tc::mbar_wait(&k_full[0], 0, err, 34);
            if (ok) {
                tc::fence_after_sync();
                issue_s(0, 0);
                if (hasB) issue_s(1, 0);
                tc::mma_commit(&k_empty[0]);
            }
            for (int j = 0; ok && j < nt; ++j) {
                const int s = j & 1;
                const uint32_t u = (uint32_t)j >> 1;
                const int n1 = j + 1;
                bool v_ok = false, k_ok = false;
                if (j < ntA) {
                    ok = tc::mbar_wait(&p_full[0], (uint32_t)j & 1u, err, 35) && tc::mbar_wait(&v_full[s], u & 1u, err, 36);
                    if (!ok) break;
                    v_ok = true;
                    tc::fence_after_sync();
                    issue_pv(0, j);
                    if (n1 < ntA) {
                        ok = tc::mbar_wait(&k_full[n1 & 1], (uint32_t)(n1 >> 1) & 1u, err, 37);
                        if (!ok) break;
                        k_ok = true;
                        tc::fence_after_sync();
                        issue_s(0, n1);
                    }
                }
                if (hasB) {
                    ok = tc::mbar_wait(&p_full[1], (uint32_t)j & 1u, err, 38) &&
                         (v_ok || tc::mbar_wait(&v_full[s], u & 1u, err, 39));
                    if (!ok) break;
                    tc::fence_after_sync();
                    issue_pv(1, j);
                    if (n1 < ntB) {
                        if (!k_ok) ok = tc::mbar_wait(&k_full[n1 & 1], (uint32_t)(n1 >> 1) & 1u, err, 40);
                        if (!ok) break;
                        tc::fence_after_sync();
                        issue_s(1, n1);
                    }
                }
                tc::mma_commit(&v_empty[s]);
                if (n1 < nt) tc::mma_commit(&k_empty[n1 & 1]);
            }
        }
    } else {
        // ---------------- softmax and output: tile t, one query row per thread ----------------
        const int t = warp >> 2, rq = warp & 3;
        const int r = rq * 32 + lane;
        const int qrow0 = q0 + t * 128;
        const int qpos = qrow0 + r;
        const uint32_t lane_base = (uint32_t)(rq * 32) << 16;
        const uint32_t tS = tmem + (uint32_t)t * 256, tO = tS + 128;
        const int ntt = t == 0 ? ntA : ntB;
        float m = -1e30f, l = 0.f;
        bool ok = true;
        for (int j = 0; ok && j < ntt; ++j) {
            ok = __all_sync(0xffffffffu, tc::mbar_wait(&s_full[t], (uint32_t)j & 1u, err, 42));
            if (!ok) break;
            tc::fence_after_sync();
            uint32_t v[128];
#pragma unroll
            for (int c = 0; c < 4; ++c)
                tc::tmem_ld32(tS + lane_base + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&v[32 * c]));
            tc::tmem_wait_ld();
            const int kbase = j * 128;
            if (kbase + 127 > qrow0 || kbase + 128 > S) {  // diagonal or ragged tile (warp-uniform)
#pragma unroll
                for (int e = 0; e < 128; ++e)
                    if (kbase + e > qpos || kbase + e >= S) v[e] = 0xff800000u;  // -inf
            }
            float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int e = 0; e < 128; ++e) mx4[e & 3] = fmaxf(mx4[e & 3], __uint_as_float(v[e]));
            const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * scale_log2;
            const float m_new = fmaxf(m, mx);
            const bool resc = m_new > m + 8.f;
            const float m_use = resc ? m_new : m;
            const float alpha = fast_exp2(m - m_use);
            if (j > 0 && __any_sync(0xffffffffu, resc)) {
                // PV_{j-1} has completed (S_j, issued behind it, has)
#pragma unroll 1
                for (int c = 0; c < D; c += 32) {
                    uint32_t o[32];
                    tc::tmem_ld32(tO + lane_base + c, o);
                    tc::tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
                    tc::tmem_st32(tO + lane_base + c, o);
                }
            }
            m = m_use;
            float l4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int c = 0; c < 128; c += 32) {
                uint32_t pk[16];
#pragma unroll
                for (int e = 0; e < 32; e += 2) {
                    const float p0 = fast_exp2(fmaf(__uint_as_float(v[c + e]), scale_log2, -m));
                    const float p1 = fast_exp2(fmaf(__uint_as_float(v[c + e + 1]), scale_log2, -m));
                    l4[(e >> 1) & 3] += p0 + p1;
                    pk[e >> 1] = pack2<BF16>(p0, p1);
                }
                tc::tmem_st16(tS + lane_base + (uint32_t)(c >> 1), pk);
            }
            l = l * alpha + ((l4[0] + l4[1]) + (l4[2] + l4[3]));
            tc::tmem_wait_st();
            tc::fence_before_sync();
            tc::mbar_arrive(&p_full[t]);
        }
        if (ok && ntt > 0) {
            const uint32_t jl = (uint32_t)(ntt - 1);
            ok = __all_sync(0xffffffffu, tc::mbar_wait(&o_done[t], jl & 1u, err, 43));
        }
        tc::fence_after_sync();
        const float inv_l = l > 0.f ? 1.f / l : 0.f;
        using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
        T* orow = static_cast<T*>(out) + ((int64_t)b * S + qpos) * ldo + (int64_t)h * D;
        if (ntt > 0) {
#pragma unroll 1
            for (int c = 0; c < D; c += 32) {
                uint32_t vv[32];
                tc::tmem_ld32(tO + lane_base + c, vv);
                tc::tmem_wait_ld();
                if (!ok || qpos >= S) continue;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    uint4 w;
                    w.x = pack2<BF16>(__uint_as_float(vv[8 * q + 0]) * inv_l, __uint_as_float(vv[8 * q + 1]) * inv_l);
                    w.y = pack2<BF16>(__uint_as_float(vv[8 * q + 2]) * inv_l, __uint_as_float(vv[8 * q + 3]) * inv_l);
                    w.z = pack2<BF16>(__uint_as_float(vv[8 * q + 4]) * inv_l, __uint_as_float(vv[8 * q + 5]) * inv_l);
                    w.w = pack2<BF16>(__uint_as_float(vv[8 * q + 6]) * inv_l, __uint_as_float(vv[8 * q + 7]) * inv_l);
                    *reinterpret_cast<uint4*>(orow + c + 8 * q) = w;
                }
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, 512);
    }
}

// Rotated-copy buffer of the RoPE form (q and k): one per device, grown on
// demand and kept (freed at process exit).  Calls with RoPE on one device
// that overlap in time (different streams) would share it and must not be
// issued.
static std::mutex g_rk_mu;
static void* g_rk_buf[64];
static size_t g_rk_bytes[64];

static int rotated_copy_buffer(size_t bytes, void** out) {
    int dev = 0;
    B2_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return B2_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lk(g_rk_mu);
    if (g_rk_bytes[dev] < bytes) {
        if (g_rk_buf[dev]) B2_TRY(cudaFree(g_rk_buf[dev]));
        g_rk_buf[dev] = nullptr;
        g_rk_bytes[dev] = 0;
        B2_TRY(cudaMalloc(&g_rk_buf[dev], bytes));
        g_rk_bytes[dev] = bytes;
    }
    *out = g_rk_buf[dev];
    return B2_OK;
}

// B2_FLASH2=0 in the environment selects the one-Q-tile kernel for head_dim 128.
static bool flash2_enabled() {
    static int on = -1;
    if (on < 0) {
        const char* e = getenv("B2_FLASH2");
        on = (e && e[0] == '0') ? 0 : 1;
    }
    return on == 1;
}

// Workspace bytes of the RoPE form: the rotated Q and K copies.
static size_t rope_copy_bytes(int64_t S, int nq, int nkv, int D, int batch) {
    return (size_t)batch * S * (nq + nkv) * D * 2;
}

template <int D, bool BF16>
static int launch_flash(const FlashArgs& a_in, cudaStream_t s) {
    using Cfg = FlashCfg<D>;
    int* err = wait_error_word();
    if (!err) return B2_ERR_STATE;
    FlashArgs a = a_in;
    if (a.rope_theta > 0.f) {  // q and k rotated once into dense copies; the tiles then come from them
        void* ws = nullptr;
        const size_t need = rope_copy_bytes(a.S, a.nq, a.nkv, D, a.batch);
        if (a.rk_ws) {  // the caller's workspace: nothing is allocated here
            if (a.rk_ws_bytes < need || !aligned16(a.rk_ws)) return B2_ERR_WORKSPACE;
            ws = a.rk_ws;
        } else {
            const int rrc = rotated_copy_buffer(need, &ws);
            if (rrc != B2_OK) return rrc;
        }
        uint16_t* qo = static_cast<uint16_t*>(ws);
        uint16_t* ko = qo + (size_t)a.batch * a.S * a.nq * D;
        const int64_t work = (int64_t)a.batch * a.S * ((a.nq + a.nkv + 7) / 8) * (D / 16);
        int64_t blocks = (work + 255) / 256;
        if (blocks > (int64_t)sm_count() * 16) blocks = (int64_t)sm_count() * 16;
        B2_TRY(launch(rope_qk_kernel<BF16>, dim3((unsigned)blocks), dim3(256), 0, s, true,
                      static_cast<const uint16_t*>(a.q), a.ldq, static_cast<const uint16_t*>(a.k), a.ldkv, qo, ko,
                      a.S, a.nq, a.nkv, D, a.batch, a.rope_theta, a.pos0));
        a.q = qo;
        a.ldq = (int64_t)a.nq * D;
        a.k = ko;
    }
    const int64_t ldk = a.rope_theta > 0.f ? (int64_t)a.nkv * D : a.ldkv;
    const CUtensorMapDataType dt = BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUtensorMap tq, tk, tv;
    const uint32_t box[4] = {64, 1, 128, 1};
    {
        const uint64_t dims[4] = {(uint64_t)D, (uint64_t)a.nq, (uint64_t)a.S, (uint64_t)a.batch};
        const uint64_t st[3] = {(uint64_t)D * 2, (uint64_t)a.ldq * 2, (uint64_t)a.S * a.ldq * 2};
        const int rc = make_tensor_map(&tq, dt, 4, a.q, dims, st, box);
        if (rc != B2_OK) return rc;
    }
    {
        const uint64_t dims[4] = {(uint64_t)D, (uint64_t)a.nkv, (uint64_t)a.S, (uint64_t)a.batch};
        const uint64_t st[3] = {(uint64_t)D * 2, (uint64_t)a.ldkv * 2, (uint64_t)a.S * a.ldkv * 2};
        const uint64_t stk[3] = {(uint64_t)D * 2, (uint64_t)ldk * 2, (uint64_t)a.S * ldk * 2};
        int rc = make_tensor_map(&tk, dt, 4, a.k, dims, stk, box);
        if (rc != B2_OK) return rc;
        rc = make_tensor_map(&tv, dt, 4, a.v, dims, st, box);
        if (rc != B2_OK) return rc;
    }
    const float scale_log2 = 1.4426950408889634f / sqrtf((float)D);
    if (D == 128 && flash2_enabled()) {
        auto kern2 = flash2_tc_kernel<BF16>;
        B2_TRY(cudaFuncSetAttribute(kern2, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)F2Cfg::SMEM));
        dim3 grid2((unsigned)a.nq, (unsigned)((a.S + 255) / 256), (unsigned)a.batch);
        B2_TRY(launch(kern2, grid2, dim3(F2Cfg::THREADS), F2Cfg::SMEM, s, true, tq, tk, tv, a.out, a.ldo, a.S, a.nq,
                      a.nkv, scale_log2, err));
        return B2_OK;
    }
    auto kern = flash_tc_kernel<D, BF16>;
    B2_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg::SMEM));
    dim3 grid((unsigned)a.nq, (unsigned)((a.S + 127) / 128), (unsigned)a.batch);
    B2_TRY(launch(kern, grid, dim3(Cfg::THREADS), Cfg::SMEM, s, true, tq, tk, tv, a.out, a.ldo, a.S, a.nq, a.nkv,
                  scale_log2, err));
    return B2_OK;
}

template <bool BF16>
static int flash_dispatch_d(const FlashArgs& a, cudaStream_t s) {
    if (a.D == 64) return launch_flash<64, BF16>(a, s);
    if (a.D == 128) return launch_flash<128, BF16>(a, s);
    return B2_ERR_UNSUPPORTED;
}

// Tensor-core flash prefill over token-major rows with explicit row strides
// (elements between consecutive tokens of q, of k/v and of out; heads are D
// apart inside a row); B2_ERR_UNSUPPORTED for shapes it does not take.
int flash_prefill_tc(const FlashArgs& a, cudaStream_t s) {
    if ((a.D != 64 && a.D != 128) || a.S <= 0 || a.S > (1 << 30) || !aligned16(a.q) || !aligned16(a.k) ||
        !aligned16(a.v) || !aligned16(a.out) || a.batch > 65535 || a.nq > 65535 || (a.ldq & 7) || (a.ldkv & 7) ||
        (a.ldo & 7))
        return B2_ERR_UNSUPPORTED;
    return a.bf16 ? flash_dispatch_d<true>(a, s) : flash_dispatch_d<false>(a, s);
}

}  // namespace b2

static b2::FlashArgs dense_args(const void* q, const void* k, const void* v, void* out, int64_t S, int nq, int nkv,
                                int D, int batch, bool bf16, float theta, int pos0) {
    b2::FlashArgs a = {};
    a.q = q;
    a.k = k;
    a.v = v;
    a.out = out;
    a.S = (int)S;
    a.nq = nq;
    a.nkv = nkv;
    a.D = D;
    a.batch = batch;
    a.ldq = (int64_t)nq * D;
    a.ldkv = (int64_t)nkv * D;
    a.ldo = (int64_t)nq * D;
    a.bf16 = bf16;
    a.rope_theta = theta;
    a.pos0 = pos0;
    return a;
}

extern "C" int b2_flash_prefill_gqa(const void* q, const void* k, const void* v, void* out, int64_t S, int nq,
                                    int nkv, int D, int batch, void* stream) {
    using namespace b2;
    if (S <= 0 || batch <= 0) return B2_OK;
    B2_REQUIRE(q && k && v && out && nq > 0 && nkv > 0 && nq % nkv == 0);
    if (S > (1 << 30)) return B2_ERR_UNSUPPORTED;
    const int rc = flash_prefill_tc(dense_args(q, k, v, out, S, nq, nkv, D, batch, false, 0.f, 0), as_stream(stream));
    if (rc != B2_ERR_UNSUPPORTED) return rc;
    if (!attn_head_dim_supported(D) || !aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
        return B2_ERR_UNSUPPORTED;
    return causal_attention_rows((const __half*)q, (const __half*)k, (const __half*)v, (__half*)out, S, nq, nkv, D,
                                 batch, as_stream(stream));
}

extern "C" int b2_flash_prefill_gqa_ex(const void* q, const void* k, const void* v, void* out, int64_t S, int nq,
                                       int nkv, int D, int batch, int bf16, float rope_theta, int64_t start_pos,
                                       void* stream) {
    return b2_flash_prefill_gqa_ws(q, k, v, out, S, nq, nkv, D, batch, bf16, rope_theta, start_pos, nullptr, stream);
}

struct b2_workspace {
    void* ptr = nullptr;
    size_t bytes = 0;
};

extern "C" int b2_workspace_create(size_t bytes, b2_workspace** out) {
    B2_REQUIRE(out && bytes > 0);
    *out = nullptr;
    b2_workspace* w = new (std::nothrow) b2_workspace();
    if (!w) return B2_ERR_INVALID;
    const cudaError_t e = cudaMalloc(&w->ptr, bytes);
    if (e != cudaSuccess) {
        delete w;
        return (int)e;
    }
    w->bytes = bytes;
    *out = w;
    return B2_OK;
}

extern "C" int b2_workspace_destroy(b2_workspace* ws) {
    if (!ws) return B2_OK;
    cudaFree(ws->ptr);
    delete ws;
    return B2_OK;
}

extern "C" size_t b2_workspace_bytes(const b2_workspace* ws) { return ws ? ws->bytes : 0; }

extern "C" size_t b2_flash_prefill_workspace_bytes(int64_t S, int num_q_heads, int num_kv_heads, int head_dim,
                                                   int batch) {
    return S > 0 && num_q_heads > 0 && num_kv_heads > 0 && head_dim > 0 && batch > 0
               ? b2::rope_copy_bytes(S, num_q_heads, num_kv_heads, head_dim, batch)
               : 0;
}

extern "C" int b2_flash_prefill_gqa_ws(const void* q, const void* k, const void* v, void* out, int64_t S, int nq,
                                       int nkv, int D, int batch, int bf16, float rope_theta, int64_t start_pos,
                                       b2_workspace* ws, void* stream) {
    using namespace b2;
    if (S <= 0 || batch <= 0) return B2_OK;
    B2_REQUIRE(q && k && v && out && nq > 0 && nkv > 0 && nq % nkv == 0 && rope_theta >= 0.f && start_pos >= 0);
    B2_REQUIRE(start_pos + S < (int64_t)1 << 24);  // positions stay exact in float
    FlashArgs a = dense_args(q, k, v, out, S, nq, nkv, D, batch, bf16 != 0, rope_theta, (int)start_pos);
    if (ws) {
        a.rk_ws = ws->ptr;
        a.rk_ws_bytes = ws->bytes;
    }
    return flash_prefill_tc(a, as_stream(stream));
}
