// gemm.cu -- C = A * B^T for the prefill projections (operator API
// matmul_transB / matmul_transB_f32), half in, fp32 accumulation.
//
// Main path: a tcgen05 kernel.  One CTA computes a 128 x BN tile of C
// (BN = 256, or 128 when 256-wide tiles would leave SMs idle).  Six warps:
//   warp 4      TMA producer: 128x64 A and BNx64 B tiles, 128-byte swizzled,
//               into a STAGES-deep shared-memory ring (full/empty mbarriers);
//   warp 5      MMA issuer: 4 tcgen05.mma (M=128, N=BN, K=16) per 64-deep k
//               block into a BN-column fp32 accumulator in TMEM, each k block
//               released to the producer by tcgen05.commit;
//   warps 0..3  epilogue: tcgen05.ld of their 32 TMEM lanes (= C rows),
//               conversion and 16-byte stores.
// Every mbarrier wait is bounded (tc.cuh).  M = 1 goes to the decode GEMV;
// shapes TMA cannot describe (K not a multiple of 8, unaligned bases) go to a
// shared-memory tiled CUDA-core kernel.
// Reference replaced: src/cuda/matmul.cu:23-79 (cublasGemmEx).
#include "tc.cuh"

namespace b2 {

// ---------------------------------------------------------------------------
// tcgen05 path
// ---------------------------------------------------------------------------
constexpr int kTcBM = 128, kTcBK = 64;

template <int BN>
struct TcGemmCfg {
    static constexpr int STAGES = BN == 256 ? 4 : 6;
    static constexpr uint32_t A_BYTES = kTcBM * kTcBK * 2;
    static constexpr uint32_t B_BYTES = BN * kTcBK * 2;
    static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
    // ring + barriers + TMEM slot, plus 1 KB to align the ring to 1024 bytes
    static constexpr size_t SMEM = (size_t)STAGES * STAGE_BYTES + 256 + 1024;
};

// Epilogue forms: half C, fp32 C, or fp32 C += A B^T (residual stream).
enum TcEpi : int { TC_HALF = 0, TC_F32 = 1, TC_F32_ADD = 2 };

template <int BN, int EPI>
__global__ void __launch_bounds__(192, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   void* __restrict__ C, int M, int N, int K, int kb_per_split, int* err) {
    using Cfg = TcGemmCfg<BN>;
    constexpr int STAGES = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* accum = empty + STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        tc::mbar_init(accum, 1);
        tc::fence_barrier_init();
    }
    if (warp == 0) tc::tmem_alloc(tmem_slot, BN);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    griddep_wait();  // A may be the previous kernel's output
    griddep_launch_dependents();

    // Tile of this CTA: tiles in groups of up to kGroupM M-tiles, the M index
    // fastest inside a group, so the CTAs in flight together share each B
    // (weight) tile and B streams through L2 once per group instead of once
    // per row of M-tiles (2048 x 4096 x 28672: 235 MB of B read once rather
    // than 16 times).
    constexpr int kGroupM = 16;
    const int tilesM = (M + kTcBM - 1) / kTcBM, tilesN = (N + BN - 1) / BN;
    const int grp = (int)blockIdx.x / (kGroupM * tilesN);
    const int gm = min(kGroupM, tilesM - grp * kGroupM);
    const int local = (int)blockIdx.x - grp * kGroupM * tilesN;
    const int m0 = (grp * kGroupM + local % gm) * kTcBM, n0 = (local / gm) * BN;
    // split-K: this CTA's k blocks [kb0, kb1); split z writes slab z of C
    const int nk_all = (K + kTcBK - 1) / kTcBK;
    const int kb0 = blockIdx.z * kb_per_split;
    const int kb1 = min(nk_all, kb0 + kb_per_split);
    const int nk = kb1 - kb0;
    if (gridDim.z > 1) C = static_cast<float*>(C) + (size_t)blockIdx.z * M * N;

    if (warp == 4) {
        if (lane == 0) {
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % STAGES;
                const uint32_t ph = (uint32_t)(kb / STAGES) & 1u;
                if (kb >= STAGES && !tc::mbar_wait(&empty[s], ph ^ 1u, err, 1)) break;
                uint8_t* st = smem + s * Cfg::STAGE_BYTES;
                tc::mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES);
                tc::tma_load_2d(st, &tmA, &full[s], (kb0 + kb) * kTcBK, m0);
                tc::tma_load_2d(st + Cfg::A_BYTES, &tmB, &full[s], (kb0 + kb) * kTcBK, n0);
            }
        }
    } else if (warp == 5) {
        if (lane == 0) {
            constexpr uint32_t idesc = tc::idesc_f16(kTcBM, BN, false, false);
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % STAGES;
                const uint32_t ph = (uint32_t)(kb / STAGES) & 1u;
                if (!tc::mbar_wait(&full[s], ph, err, 2)) break;
                tc::fence_after_sync();
                const uint32_t a = tc::smem_u32(smem + s * Cfg::STAGE_BYTES);
                const uint32_t b = a + Cfg::A_BYTES;
#pragma unroll
                for (int k = 0; k < kTcBK / 16; ++k)
                    tc::mma_f16(tmem, tc::desc_k_sw128(a + 32 * k), tc::desc_k_sw128(b + 32 * k), idesc,
                                (kb | k) != 0 ? 1u : 0u);
                tc::mma_commit(&empty[s]);
            }
            tc::mma_commit(accum);
        }
    } else {
        // epilogue: warp w owns TMEM lanes / C rows 32w .. 32w+31
        const bool ok = tc::mbar_wait(accum, 0, err, 3);
        tc::fence_after_sync();
        const int row = m0 + warp * 32 + lane;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
            uint32_t r[32];
            tc::tmem_ld32(tc::taddr(tmem, warp * 32, c), r);
            tc::tmem_wait_ld();
            if (!ok || row >= M || n0 + c >= N) continue;
            const int ncol = min(32, N - (n0 + c));
            if constexpr (EPI == TC_F32_ADD) {
                float* dst = static_cast<float*>(C) + (size_t)row * N + n0 + c;
                if (ncol == 32 && (N & 3) == 0) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        float4 o = *reinterpret_cast<float4*>(dst + j);
                        o.x += __uint_as_float(r[j]);
                        o.y += __uint_as_float(r[j + 1]);
                        o.z += __uint_as_float(r[j + 2]);
                        o.w += __uint_as_float(r[j + 3]);
                        *reinterpret_cast<float4*>(dst + j) = o;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (j < ncol) dst[j] += __uint_as_float(r[j]);
                }
            } else if constexpr (EPI == TC_F32) {
                float* dst = static_cast<float*>(C) + (size_t)row * N + n0 + c;
                if (ncol == 32 && (N & 3) == 0) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        *reinterpret_cast<uint4*>(dst + j) = make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (j < ncol) dst[j] = __uint_as_float(r[j]);
                }
            } else {
                __half* dst = static_cast<__half*>(C) + (size_t)row * N + n0 + c;
                if (ncol == 32 && (N & 7) == 0) {
#pragma unroll
                    for (int j = 0; j < 32; j += 8) {
                        float f[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(r[j + e]);
                        *reinterpret_cast<uint4*>(dst + j) = pack8(f);
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (j < ncol) dst[j] = __float2half_rn(__uint_as_float(r[j]));
                }
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, BN);
    }
}

template <int BN, int EPI>
static int launch_tc(const CUtensorMap& ta, const CUtensorMap& tb, void* C, int M, int N, int K, int ksplit,
                     int* err, cudaStream_t s) {
    auto kern = gemm_tc_kernel<BN, EPI>;
    const size_t smem = TcGemmCfg<BN>::SMEM;
    B2_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int nk = (K + kTcBK - 1) / kTcBK;
    const int kbps = (nk + ksplit - 1) / ksplit;
    ksplit = (nk + kbps - 1) / kbps;  // no empty split
    dim3 grid((unsigned)(((N + BN - 1) / BN) * ((M + kTcBM - 1) / kTcBM)), 1u, (unsigned)ksplit);
    B2_TRY(launch(kern, grid, dim3(192), smem, s, true, ta, tb, C, M, N, K, kbps, err));
    return B2_OK;
}

template <int BN>
static int launch_tc_epi(const CUtensorMap& ta, const CUtensorMap& tb, void* C, int M, int N, int K, int epi,
                         int ksplit, int* err, cudaStream_t s) {
    switch (epi) {
        case TC_HALF: return launch_tc<BN, TC_HALF>(ta, tb, C, M, N, K, 1, err, s);
        case TC_F32: return launch_tc<BN, TC_F32>(ta, tb, C, M, N, K, ksplit, err, s);
        default: return launch_tc<BN, TC_F32_ADD>(ta, tb, C, M, N, K, 1, err, s);
    }
}

// C[M,N] (=, or += for TC_F32_ADD) A[M,K] * B[N,K]^T on the tensor cores.
// Requires 16-byte aligned A, B, C and K % 8 == 0 (TMA row strides are
// multiples of 16 bytes); B2_ERR_UNSUPPORTED otherwise.  ksplit > 1 (TC_F32
// only): the K range is cut into that many parts (at most; whole 64-deep
// blocks each) and part z writes fp32 slab z of C ([ksplit][M][N]) for the
// caller to reduce; the number of slabs written is returned through
// *slabs when it is not null.
int gemm_tc_split(const __half* A, const __half* B, void* C, int M, int N, int K, int epi, int ksplit, int* slabs,
                  cudaStream_t s);

int gemm_tc(const __half* A, const __half* B, void* C, int M, int N, int K, int epi, cudaStream_t s) {
    return gemm_tc_split(A, B, C, M, N, K, epi, 1, nullptr, s);
}

int gemm_tc_split(const __half* A, const __half* B, void* C, int M, int N, int K, int epi, int ksplit, int* slabs,
                  cudaStream_t s) {
    if (ksplit > 1 && epi != TC_F32) return B2_ERR_INVALID;
    if (ksplit < 1) ksplit = 1;
    {
        const int nk = (K + kTcBK - 1) / kTcBK;
        const int kbps = (nk + ksplit - 1) / ksplit;
        if (slabs) *slabs = (nk + kbps - 1) / kbps;
    }
    if (M <= 0 || N <= 0 || K <= 0) return B2_ERR_UNSUPPORTED;
    if ((K & 7) || !aligned16(A) || !aligned16(B) || !aligned16(C)) return B2_ERR_UNSUPPORTED;
    int* err = wait_error_word();
    if (!err) return B2_ERR_STATE;
    const int tiles256 = ((N + 255) / 256) * ((M + kTcBM - 1) / kTcBM);
    const int BN = tiles256 >= sm_count() ? 256 : 128;
    CUtensorMap ta, tb;
    const uint64_t da[2] = {(uint64_t)K, (uint64_t)M}, sa[1] = {(uint64_t)K * 2};
    const uint32_t ba[2] = {(uint32_t)kTcBK, (uint32_t)kTcBM};
    const uint64_t db[2] = {(uint64_t)K, (uint64_t)N}, sb[1] = {(uint64_t)K * 2};
    const uint32_t bb[2] = {(uint32_t)kTcBK, (uint32_t)BN};
    int rc = make_tensor_map(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, A, da, sa, ba);
    if (rc != B2_OK) return rc;
    rc = make_tensor_map(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, B, db, sb, bb);
    if (rc != B2_OK) return rc;
    return BN == 256 ? launch_tc_epi<256>(ta, tb, C, M, N, K, epi, ksplit, err, s)
                     : launch_tc_epi<128>(ta, tb, C, M, N, K, epi, ksplit, err, s);
}

// ---------------------------------------------------------------------------
// generic path: shared-memory tiled CUDA-core kernel for shapes TMA cannot
// describe.  64x64 output tile per CTA, 16-deep k slabs, 4x4 outputs per thread.
// ---------------------------------------------------------------------------
constexpr int TM = 64, TN = 64, TK = 16;

template <bool OUT_F32>
__global__ void __launch_bounds__(256) gemm_tn_kernel(const __half* __restrict__ A, const __half* __restrict__ B,
                                                      void* __restrict__ C, int M, int K, int N) {
    __shared__ float As[TK][TM + 4];
    __shared__ float Bs[TK][TN + 4];
    griddep_wait();
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += TK) {
        for (int i = threadIdx.x; i < TM * TK; i += 256) {
            const int r = i / TK, kk = i - (i / TK) * TK;
            const int gm = m0 + r, gk = k0 + kk;
            As[kk][r] = (gm < M && gk < K) ? __half2float(A[(size_t)gm * K + gk]) : 0.f;
            const int gn = n0 + r;
            Bs[kk][r] = (gn < N && gk < K) ? __half2float(B[(size_t)gn * K + gk]) : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < TK; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int gm = m0 + ty * 4 + i;
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int gn = n0 + tx * 4 + j;
            if (gn >= N) continue;
            if (OUT_F32) static_cast<float*>(C)[(size_t)gm * N + gn] = acc[i][j];
            else static_cast<__half*>(C)[(size_t)gm * N + gn] = __float2half_rn(acc[i][j]);
        }
    }
}

static int gemm_api(const void* A, const void* B, void* C, int M, int K, int N, bool f32, void* stream) {
    if (M <= 0 || N <= 0) return B2_OK;
    B2_REQUIRE(A && B && C && K >= 0);
    cudaStream_t s = as_stream(stream);
    if (M == 1 && K > 0) return b2_gemv_batched(B, A, nullptr, C, 1, N, K, 0, f32 ? 1 : 0, stream);
    if (K > 0) {
        const int rc = gemm_tc((const __half*)A, (const __half*)B, C, M, N, K, f32 ? TC_F32 : TC_HALF, s);
        if (rc != B2_ERR_UNSUPPORTED) return rc;
    }
    dim3 grid((unsigned)((N + TN - 1) / TN), (unsigned)((M + TM - 1) / TM));
    if (f32)
        B2_TRY(launch(gemm_tn_kernel<true>, grid, dim3(256), 0, s, true, (const __half*)A, (const __half*)B, C, M, K, N));
    else
        B2_TRY(launch(gemm_tn_kernel<false>, grid, dim3(256), 0, s, true, (const __half*)A, (const __half*)B, C, M, K, N));
    return B2_OK;
}

}  // namespace b2

extern "C" int b2_matmul_transB(const void* A, const void* B, void* C, int M, int K, int N, void* stream) {
    return b2::gemm_api(A, B, C, M, K, N, false, stream);
}

extern "C" int b2_matmul_transB_f32(const void* A, const void* B, float* C, int M, int K, int N, void* stream) {
    return b2::gemm_api(A, B, C, M, K, N, true, stream);
}
