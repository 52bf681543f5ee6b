/*
 * b2oracle.c -- CPU restatement of the reference engine's per-token forward
 * path (XVX-016/serving-engine, src/cpu + src/model/forward_cpu + the host
 * tail of src/runtime/sampler.cu).
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA path is
 * compared against.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / reference legs load it.  The product library never links or
 * calls it.
 *
 * Parity is pinned two ways:
 *   - against the known-answer cases of the reference's tests/test_cpu_ops.cpp
 *     (restated in tests/test_oracle.py), and
 *   - against the reference's own src/cpu + forward_cpu compiled from its
 *     sources into oracle/_ref (tests/test_oracle.py), with committed
 *     golden vectors under tests/golden generated from that build.
 *
 * Every function keeps the reference's accumulation order (double partial sums
 * per 64-wide k block folded into float, float softmax, float RoPE with
 * glibc powf/cosf/sinf), so on the same host its outputs are bit-identical to
 * the reference's.  Work is split across pthreads by output row only, which
 * leaves each output's arithmetic untouched.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* threading                                                                */
/* ------------------------------------------------------------------------ */

static int g_threads = 1;

void ora_set_threads(int n) { g_threads = n < 1 ? 1 : (n > 512 ? 512 : n); }
int ora_get_threads(void) { return g_threads; }

typedef void (*ora_range_fn)(void* ctx, int64_t begin, int64_t end);

typedef struct {
    ora_range_fn fn;
    void* ctx;
    int64_t begin, end;
} ora_job;

static void* ora_job_main(void* p) {
    ora_job* j = (ora_job*)p;
    if (j->begin < j->end) j->fn(j->ctx, j->begin, j->end);
    return NULL;
}

/* Run fn over [0, n) split into contiguous slices, one per thread. */
static void ora_parallel_for(int64_t n, int64_t min_per_thread, ora_range_fn fn, void* ctx) {
    int t = g_threads;
    if (min_per_thread < 1) min_per_thread = 1;
    if ((int64_t)t > n / min_per_thread) t = (int)(n / min_per_thread);
    if (t <= 1) {
        fn(ctx, 0, n);
        return;
    }
    pthread_t th[512];
    ora_job jobs[512];
    int64_t per = (n + t - 1) / t;
    for (int i = 0; i < t; ++i) {
        jobs[i].fn = fn;
        jobs[i].ctx = ctx;
        jobs[i].begin = i * per;
        jobs[i].end = (i + 1) * per < n ? (i + 1) * per : n;
    }
    for (int i = 1; i < t; ++i) pthread_create(&th[i], NULL, ora_job_main, &jobs[i]);
    ora_job_main(&jobs[0]);
    for (int i = 1; i < t; ++i) pthread_join(th[i], NULL);
}

/* ------------------------------------------------------------------------ */
/* fp16 helpers (IEEE binary16, round-to-nearest-even via _Float16)          */
/* ------------------------------------------------------------------------ */

void ora_f32_to_f16(const float* src, uint16_t* dst, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        _Float16 h = (_Float16)src[i];
        memcpy(&dst[i], &h, 2);
    }
}

void ora_f16_to_f32(const uint16_t* src, float* dst, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        _Float16 h;
        memcpy(&h, &src[i], 2);
        dst[i] = (float)h;
    }
}

/* ------------------------------------------------------------------------ */
/* seeded weight generator shared bit-for-bit with the device init kernel    */
/* (serving-engine_b200/csrc/model.cu, init_tensor_kernel)                   */
/* ------------------------------------------------------------------------ */

static inline uint64_t ora_mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* Scale that maps an Irwin-Hall sum of four 16-bit uniforms to unit variance,
 * times the requested std.  Computed once on the host in double, then used as
 * a float on both sides. */
float ora_init_scale(double stddev) {
    double var1 = (65536.0 * 65536.0 - 1.0) / 12.0;
    return (float)(stddev / sqrt(4.0 * var1));
}

/* Element `index` of tensor `tensor_id`: approximately N(0, std^2) (Irwin-Hall
 * sum of four uniforms, exact integer arithmetic), one float multiply, rounded
 * to fp16.  Returns raw fp16 bits. */
uint16_t ora_init_value(uint64_t seed, uint64_t tensor_id, uint64_t index, float scale) {
    uint64_t key = ora_mix64(seed + 0x9E3779B97F4A7C15ull * (tensor_id + 1));
    uint64_t r = ora_mix64(key ^ index);
    int32_t s = (int32_t)(r & 0xFFFF) + (int32_t)((r >> 16) & 0xFFFF) +
                (int32_t)((r >> 32) & 0xFFFF) + (int32_t)((r >> 48) & 0xFFFF);
    volatile float v = (float)(s - 131070) * scale; /* single rounding, no FMA */
    _Float16 h = (_Float16)v;
    uint16_t bits;
    memcpy(&bits, &h, 2);
    return bits;
}

typedef struct {
    uint64_t seed, tensor_id;
    int64_t rows_total_offset, cols, col_offset, ld_global;
    float scale;
    uint16_t* out;
} ora_init_ctx;

static void ora_init_rows(void* p, int64_t b, int64_t e) {
    ora_init_ctx* c = (ora_init_ctx*)p;
    const uint64_t key = ora_mix64(c->seed + 0x9E3779B97F4A7C15ull * (c->tensor_id + 1));
    for (int64_t r = b; r < e; ++r) {
        uint64_t grow = (uint64_t)(r + c->rows_total_offset);
        for (int64_t j = 0; j < c->cols; ++j) {
            uint64_t idx = grow * (uint64_t)c->ld_global + (uint64_t)(j + c->col_offset);
            uint64_t h = ora_mix64(key ^ idx);
            int32_t s = (int32_t)(h & 0xFFFF) + (int32_t)((h >> 16) & 0xFFFF) +
                        (int32_t)((h >> 32) & 0xFFFF) + (int32_t)((h >> 48) & 0xFFFF);
            float v = (float)(s - 131070) * c->scale;
            _Float16 hv = (_Float16)v;
            memcpy(&c->out[r * c->cols + j], &hv, 2);
        }
    }
}

/* Fill a [rows, cols] fp16 block that is the sub-block starting at global
 * (row_offset, col_offset) of a tensor whose global row length is ld_global. */
void ora_init_tensor(uint64_t seed, uint64_t tensor_id, int64_t rows, int64_t cols,
                     int64_t row_offset, int64_t col_offset, int64_t ld_global,
                     float scale, uint16_t* out) {
    ora_init_ctx c = {seed, tensor_id, row_offset, cols, col_offset, ld_global, scale, out};
    ora_parallel_for(rows, 16, ora_init_rows, &c);
}

typedef struct {
    const uint16_t* src;
    float* dst;
} ora_cvt_ctx;

static void ora_cvt_range(void* p, int64_t b, int64_t e) {
    ora_cvt_ctx* c = (ora_cvt_ctx*)p;
    ora_f16_to_f32(c->src + b, c->dst + b, e - b);
}

/* fp16 -> fp32 widening split across the oracle's threads. */
void ora_f16_to_f32_par(const uint16_t* src, float* dst, int64_t n) {
    ora_cvt_ctx c = {src, dst};
    ora_parallel_for(n, 1 << 16, ora_cvt_range, &c);
}

/* ------------------------------------------------------------------------ */
/* ops  (reference: src/cpu/ops.cpp)                                         */
/* ------------------------------------------------------------------------ */

/* src/cpu/ops.cpp:11-24 */
void ora_embedding_lookup(const int64_t* ids, const float* table, float* out,
                          int64_t seq_len, int64_t hidden) {
    for (int64_t i = 0; i < seq_len; ++i)
        memcpy(out + i * hidden, table + ids[i] * hidden, (size_t)hidden * sizeof(float));
}

/* src/cpu/ops.cpp:26-51: double sum of squares, float scale, (x*r)*w */
void ora_rmsnorm(const float* x, const float* w, float* out, int64_t rows, int64_t dim, float eps) {
    for (int64_t r = 0; r < rows; ++r) {
        const float* xr = x + r * dim;
        float* o = out + r * dim;
        double ss = 0.0;
        for (int64_t c = 0; c < dim; ++c) {
            double v = (double)xr[c];
            ss += v * v;
        }
        double mean = ss / (double)dim;
        float rs = (float)(1.0 / sqrt(mean + (double)eps));
        for (int64_t c = 0; c < dim; ++c) o[c] = xr[c] * rs * w[c];
    }
}

/* src/cpu/ops.cpp:53-74 */
void ora_matmul_transB_naive(const float* A, const float* B, float* C, int64_t M, int64_t K, int64_t N) {
    for (int64_t m = 0; m < M; ++m)
        for (int64_t n = 0; n < N; ++n) {
            double s = 0.0;
            for (int64_t k = 0; k < K; ++k) s += (double)A[m * K + k] * (double)B[n * K + k];
            C[m * N + n] = (float)s;
        }
}

typedef struct {
    const float *A, *B;
    float* C;
    int64_t M, K, N;
} ora_mm_ctx;

/* One output column range n in [b, e) for all rows m.  Per output element the
 * arithmetic is exactly the reference's: C starts at 0.0f, and for each 64-wide
 * k block a double partial sum is rounded to float and added
 * (src/cpu/ops.cpp:76-114; the m/n blocking there does not change the
 * per-element order). */
static void ora_mm_cols(void* p, int64_t b, int64_t e) {
    ora_mm_ctx* c = (ora_mm_ctx*)p;
    const int64_t BK = 64;
    for (int64_t m = 0; m < c->M; ++m) {
        const float* a = c->A + m * c->K;
        for (int64_t n = b; n < e; ++n) {
            const float* bb = c->B + n * c->K;
            float acc = 0.0f;
            for (int64_t k0 = 0; k0 < c->K; k0 += BK) {
                int64_t k1 = k0 + BK < c->K ? k0 + BK : c->K;
                double s = 0.0;
                for (int64_t k = k0; k < k1; ++k) s += (double)a[k] * (double)bb[k];
                acc += (float)s;
            }
            c->C[m * c->N + n] = acc;
        }
    }
}

void ora_matmul_transB_blocked(const float* A, const float* B, float* C, int64_t M, int64_t K, int64_t N) {
    ora_mm_ctx c = {A, B, C, M, K, N};
    ora_parallel_for(N, 8, ora_mm_cols, &c);
}

/* src/cpu/ops.cpp:138-152 */
void ora_bias_add(const float* x, const float* bias, float* out, int64_t M, int64_t N) {
    for (int64_t m = 0; m < M; ++m)
        for (int64_t n = 0; n < N; ++n) out[m * N + n] = x[m * N + n] + bias[n];
}

/* src/cpu/ops.cpp:154-163 */
void ora_residual_add(const float* a, const float* b, float* out, int64_t count) {
    for (int64_t i = 0; i < count; ++i) out[i] = a[i] + b[i];
}

/* The float cos/sin table of src/cpu/ops.cpp:174-189: inv_freq =
 * 1/powf(theta, 2i/D), angle = (float)pos * inv_freq, cosf/sinf.  Rows are
 * positions [pos0, pos0 + npos), columns i in [0, D/2).  The product path uses
 * the same table (computed on the host at model creation). */
void ora_rope_table(int64_t pos0, int64_t npos, int64_t head_dim, float theta, float* cos_out, float* sin_out) {
    int64_t half = head_dim / 2;
    float* inv = (float*)malloc(sizeof(float) * (size_t)(half > 0 ? half : 1));
    for (int64_t i = 0; i < half; ++i)
        inv[i] = 1.0f / powf(theta, (float)(2 * i) / (float)head_dim);
    for (int64_t p = 0; p < npos; ++p)
        for (int64_t i = 0; i < half; ++i) {
            float a = (float)(pos0 + p) * inv[i];
            cos_out[p * half + i] = cosf(a);
            sin_out[p * half + i] = sinf(a);
        }
    free(inv);
}

/* src/cpu/ops.cpp:165-221: rotate-half RoPE, in place on q and k */
void ora_apply_rope(float* q, float* k, int64_t S, int64_t nq, int64_t nkv, int64_t D,
                    int64_t start_pos, float theta) {
    int64_t half = D / 2;
    if (S <= 0 || half <= 0) return;
    float* cs = (float*)malloc(sizeof(float) * (size_t)half);
    float* sn = (float*)malloc(sizeof(float) * (size_t)half);
    for (int64_t s = 0; s < S; ++s) {
        ora_rope_table(start_pos + s, 1, D, theta, cs, sn);
        for (int64_t h = 0; h < nq; ++h) {
            float* v = q + (s * nq + h) * D;
            for (int64_t i = 0; i < half; ++i) {
                float x1 = v[i], x2 = v[half + i];
                v[i] = x1 * cs[i] - x2 * sn[i];
                v[half + i] = x2 * cs[i] + x1 * sn[i];
            }
        }
        for (int64_t h = 0; h < nkv; ++h) {
            float* v = k + (s * nkv + h) * D;
            for (int64_t i = 0; i < half; ++i) {
                float x1 = v[i], x2 = v[half + i];
                v[i] = x1 * cs[i] - x2 * sn[i];
                v[half + i] = x2 * cs[i] + x1 * sn[i];
            }
        }
    }
    free(cs);
    free(sn);
}

typedef struct {
    const float *q, *k, *v;
    float* out;
    int64_t S, nq, nkv, D, q_begin; /* q rows [q_begin, S) */
} ora_attn_ctx;

/* src/cpu/ops.cpp:223-284, one (q head, query row) unit per index. */
static void ora_attn_units(void* p, int64_t b, int64_t e) {
    ora_attn_ctx* c = (ora_attn_ctx*)p;
    int64_t group = c->nq / c->nkv;
    float scale = 1.0f / sqrtf((float)c->D);
    int64_t rows = c->S - c->q_begin;
    float* scores = (float*)malloc(sizeof(float) * (size_t)c->S);
    for (int64_t u = b; u < e; ++u) {
        int64_t qh = u / rows;
        int64_t i = c->q_begin + u % rows;
        int64_t kvh = qh / group;
        const float* qv = c->q + (i * c->nq + qh) * c->D;
        float mx = -1e30f;
        for (int64_t j = 0; j <= i; ++j) {
            const float* kv = c->k + (j * c->nkv + kvh) * c->D;
            double dot = 0.0;
            for (int64_t d = 0; d < c->D; ++d) dot += (double)qv[d] * (double)kv[d];
            float sc = (float)dot * scale;
            scores[j] = sc;
            if (sc > mx) mx = sc;
        }
        double sum = 0.0;
        for (int64_t j = 0; j <= i; ++j) {
            float ev = expf(scores[j] - mx);
            scores[j] = ev;
            sum += (double)ev;
        }
        float inv = (float)(1.0 / sum);
        for (int64_t j = 0; j <= i; ++j) scores[j] *= inv;
        float* ov = c->out + (i * c->nq + qh) * c->D;
        for (int64_t d = 0; d < c->D; ++d) {
            double acc = 0.0;
            for (int64_t j = 0; j <= i; ++j)
                acc += (double)scores[j] * (double)c->v[(j * c->nkv + kvh) * c->D + d];
            ov[d] = (float)acc;
        }
    }
    free(scores);
}

void ora_causal_gqa_rows(const float* q, const float* k, const float* v, float* out, int64_t S,
                         int64_t nq, int64_t nkv, int64_t D, int64_t q_begin) {
    if (S <= 0 || q_begin >= S) return;
    ora_attn_ctx c = {q, k, v, out, S, nq, nkv, D, q_begin};
    ora_parallel_for(nq * (S - q_begin), 1, ora_attn_units, &c);
}

void ora_causal_gqa(const float* q, const float* k, const float* v, float* out, int64_t S,
                    int64_t nq, int64_t nkv, int64_t D) {
    ora_causal_gqa_rows(q, k, v, out, S, nq, nkv, D, 0);
}

/* src/cpu/ops.cpp:286-298 */
void ora_swiglu(const float* gate, const float* up, float* out, int64_t count) {
    for (int64_t i = 0; i < count; ++i) {
        float g = gate[i];
        float sg = g / (1.0f + expf(-g));
        out[i] = sg * up[i];
    }
}

/* Row softmax with the reference GPU kernel's semantics (src/cuda/softmax.cu:25-83:
 * max, sum of exp(x - max), e * (1/sum)), evaluated in double and rounded. */
void ora_softmax(const float* x, float* out, int64_t rows, int64_t cols) {
    for (int64_t r = 0; r < rows; ++r) {
        const float* xr = x + r * cols;
        double mx = -1e300;
        for (int64_t c = 0; c < cols; ++c) mx = xr[c] > mx ? xr[c] : mx;
        double s = 0.0;
        for (int64_t c = 0; c < cols; ++c) s += exp((double)xr[c] - mx);
        for (int64_t c = 0; c < cols; ++c) out[r * cols + c] = (float)(exp((double)xr[c] - mx) / s);
    }
}

/* Single-query decode attention over a strided KV view, as the reference's
 * kernel tests state it (tests/test_attention.cpp:79-118): float dot, float
 * max, expf, float sum, normalised weights times V.  Views are element strides
 * (b, h, s) with d contiguous.  q/out: [B, nq, D]. */
void ora_decode_attention(const float* q, const float* kbase, const float* vbase,
                          int64_t sb, int64_t sh, int64_t ss, const int* seq_lens, float* out,
                          int64_t B, int64_t nq, int64_t nkv, int64_t D) {
    int64_t group = nq / nkv;
    float scale = 1.0f / sqrtf((float)D);
    int64_t maxlen = 0;
    for (int64_t b = 0; b < B; ++b) maxlen = seq_lens[b] > maxlen ? seq_lens[b] : maxlen;
    float* sc = (float*)malloc(sizeof(float) * (size_t)(maxlen > 0 ? maxlen : 1));
    for (int64_t b = 0; b < B; ++b) {
        int64_t L = seq_lens[b];
        for (int64_t h = 0; h < nq; ++h) {
            int64_t kvh = h / group;
            const float* qv = q + (b * nq + h) * D;
            float* ov = out + (b * nq + h) * D;
            for (int64_t d = 0; d < D; ++d) ov[d] = 0.0f;
            if (L <= 0) continue;
            float mx = -1e20f;
            for (int64_t t = 0; t < L; ++t) {
                const float* kv = kbase + b * sb + kvh * sh + t * ss;
                float dot = 0.0f;
                for (int64_t d = 0; d < D; ++d) dot += qv[d] * kv[d];
                sc[t] = dot * scale;
                if (sc[t] > mx) mx = sc[t];
            }
            float sum = 0.0f;
            for (int64_t t = 0; t < L; ++t) {
                sc[t] = expf(sc[t] - mx);
                sum += sc[t];
            }
            for (int64_t t = 0; t < L; ++t) sc[t] /= sum;
            for (int64_t d = 0; d < D; ++d) {
                float acc = 0.0f;
                for (int64_t t = 0; t < L; ++t) acc += sc[t] * vbase[b * sb + kvh * sh + t * ss + d];
                ov[d] = acc;
            }
        }
    }
    free(sc);
}

/* ------------------------------------------------------------------------ */
/* full forward  (reference: src/model/forward_cpu.cpp:58-174)               */
/* ------------------------------------------------------------------------ */

typedef struct {
    int64_t vocab, hidden, inter, layers, nq, nkv, head_dim;
    float eps, theta;
    int tied;     /* 1: lm_head is the embedding table (forward_cpu.cpp:165-167) */
    int has_bias; /* 1: q/k/v biases present (Qwen2); 0: Llama, treated as zero */
} ora_config;

/* Per-layer fp32 weights, in the reference's ModelWeightsFP32::LayerFP32 order
 * (src/model/forward_cpu.h:18-38). */
typedef struct {
    const float *ln1, *ln2, *wq, *bq, *wk, *bk, *wv, *bv, *wo, *wg, *wu, *wd;
} ora_layer;

typedef struct {
    const float* embed;
    const float* final_norm;
    const float* lm_head; /* ignored when tied */
    const ora_layer* layers;
} ora_weights;

/* Full-recompute forward over S tokens.  Logits are produced for positions
 * [logit_row0, S) into logits[(S - logit_row0) * V]; each logit row is
 * bit-identical to the reference's full [S, V] output row (rows are
 * independent in matmul_transB_blocked).  Optional dumps:
 * final_hidden [S*H] (post final norm). */
int ora_forward(const ora_config* cfg, const ora_weights* w, const int64_t* ids, int64_t S,
                int64_t logit_row0, float* logits, float* final_norm_out) {
    int64_t H = cfg->hidden, D = cfg->head_dim, kvd = cfg->nkv * D, I = cfg->inter, V = cfg->vocab;
    int64_t qd = cfg->nq * D;
    if (S <= 0 || logit_row0 < 0 || logit_row0 > S) return -1;
    float* h = (float*)malloc(sizeof(float) * (size_t)(S * H));
    float* xn = (float*)malloc(sizeof(float) * (size_t)(S * H));
    float* q = (float*)malloc(sizeof(float) * (size_t)(S * qd));
    float* k = (float*)malloc(sizeof(float) * (size_t)(S * kvd));
    float* v = (float*)malloc(sizeof(float) * (size_t)(S * kvd));
    float* ao = (float*)malloc(sizeof(float) * (size_t)(S * qd));
    float* po = (float*)malloc(sizeof(float) * (size_t)(S * H));
    float* g = (float*)malloc(sizeof(float) * (size_t)(S * I));
    float* u = (float*)malloc(sizeof(float) * (size_t)(S * I));
    float* a = (float*)malloc(sizeof(float) * (size_t)(S * I));
    if (!h || !xn || !q || !k || !v || !ao || !po || !g || !u || !a) return -2;

    ora_embedding_lookup(ids, w->embed, h, S, H);
    for (int64_t l = 0; l < cfg->layers; ++l) {
        const ora_layer* L = &w->layers[l];
        ora_rmsnorm(h, L->ln1, xn, S, H, cfg->eps);
        ora_matmul_transB_blocked(xn, L->wq, q, S, H, qd);
        if (cfg->has_bias) ora_bias_add(q, L->bq, q, S, qd);
        ora_matmul_transB_blocked(xn, L->wk, k, S, H, kvd);
        if (cfg->has_bias) ora_bias_add(k, L->bk, k, S, kvd);
        ora_matmul_transB_blocked(xn, L->wv, v, S, H, kvd);
        if (cfg->has_bias) ora_bias_add(v, L->bv, v, S, kvd);
        ora_apply_rope(q, k, S, cfg->nq, cfg->nkv, D, 0, cfg->theta);
        ora_causal_gqa(q, k, v, ao, S, cfg->nq, cfg->nkv, D);
        ora_matmul_transB_blocked(ao, L->wo, po, S, qd, H);
        ora_residual_add(h, po, h, S * H);
        ora_rmsnorm(h, L->ln2, xn, S, H, cfg->eps);
        ora_matmul_transB_blocked(xn, L->wg, g, S, H, I);
        ora_matmul_transB_blocked(xn, L->wu, u, S, H, I);
        ora_swiglu(g, u, a, S * I);
        ora_matmul_transB_blocked(a, L->wd, po, S, I, H);
        ora_residual_add(h, po, h, S * H);
    }
    ora_rmsnorm(h, w->final_norm, xn, S, H, cfg->eps);
    if (final_norm_out) memcpy(final_norm_out, xn, sizeof(float) * (size_t)(S * H));
    if (logits && logit_row0 < S) {
        const float* head = cfg->tied ? w->embed : w->lm_head;
        ora_matmul_transB_blocked(xn + logit_row0 * H, head, logits, S - logit_row0, H, V);
    }
    free(h); free(xn); free(q); free(k); free(v); free(ao); free(po); free(g); free(u); free(a);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* sampler  (reference: src/runtime/sampler.cu:13-33, 36-73, 202-339)        */
/* ------------------------------------------------------------------------ */

/* Padded-vocabulary rule of src/runtime/sampler.cu:231-248,257-262: ids at or
 * above 151665 are excluded whenever the vocabulary is larger than that. */
#define ORA_REAL_VOCAB 151665

/* Repetition penalty, once per distinct id in history (sampler.cu:13-33
 * applies it per history entry with a race on duplicates; applying it once per
 * distinct id is the race-free reading). */
void ora_repetition_penalty(float* logits, int64_t V, const int64_t* hist, int64_t n, float penalty) {
    for (int64_t i = 0; i < n; ++i) {
        int64_t t = hist[i];
        if (t < 0 || t >= V) continue;
        int dup = 0;
        for (int64_t j = 0; j < i; ++j)
            if (hist[j] == t) { dup = 1; break; }
        if (dup) continue;
        float l = logits[t];
        logits[t] = l > 0.0f ? l / penalty : l * penalty;
    }
}

/* Greedy argmax over the active vocabulary; ties go to the lowest id. */
int64_t ora_argmax(const float* logits, int64_t V) {
    int64_t active = V > ORA_REAL_VOCAB ? ORA_REAL_VOCAB : V;
    int64_t best = 0;
    float bv = logits[0];
    for (int64_t i = 1; i < active; ++i)
        if (logits[i] > bv) { bv = logits[i]; best = i; }
    return best;
}

/* One LCG step of sampler.cu:321-328, returning the uniform in [0,1). */
float ora_lcg_next(uint64_t* state) {
    *state = *state * 6364136223846793005ull + 1442695040888963407ull;
    return (float)((double)(*state >> 40) * (1.0 / 16777216.0));
}

/* sampler.cu:322-324: reseed only when seed != 0 and seed != current state */
void ora_lcg_reseed(uint64_t* state, uint64_t seed) {
    if (seed != 0 && seed != *state) *state = seed;
}

static const float* g_sort_vals;
static int ora_cmp_desc(const void* a, const void* b) {
    int64_t ia = *(const int64_t*)a, ib = *(const int64_t*)b;
    float va = g_sort_vals[ia], vb = g_sort_vals[ib];
    if (va > vb) return -1;
    if (va < vb) return 1;
    return ia < ib ? -1 : (ia > ib ? 1 : 0);
}

/* Top-k / temperature / top-p / LCG draw of sampler.cu:251-339 on host logits
 * (already penalised).  K <= 0 or K > max_top_k -> min(max_top_k, 64).
 * Ties in the top-k order go to the lower id.  `u` is the LCG uniform.
 * Returns the selected id. */
int64_t ora_sample_topk_topp(const float* logits_in, int64_t V, int top_k, int max_top_k,
                             float temperature, float top_p, float u) {
    float* lg = (float*)malloc(sizeof(float) * (size_t)V);
    memcpy(lg, logits_in, sizeof(float) * (size_t)V);
    if (V > ORA_REAL_VOCAB)
        for (int64_t i = ORA_REAL_VOCAB; i < V; ++i) lg[i] = -1e9f;
    int64_t K = top_k;
    if (K <= 0 || K > max_top_k) K = max_top_k < 64 ? max_top_k : 64;
    if (K > V) K = V;
    int64_t* idx = (int64_t*)malloc(sizeof(int64_t) * (size_t)V);
    for (int64_t i = 0; i < V; ++i) idx[i] = i;
    g_sort_vals = lg;
    qsort(idx, (size_t)V, sizeof(int64_t), ora_cmp_desc);
    float maxv = lg[idx[0]] / temperature;
    float* pr = (float*)malloc(sizeof(float) * (size_t)K);
    float sum = 0.0f;
    for (int64_t i = 0; i < K; ++i) {
        float val = lg[idx[i]] / temperature;
        float e = expf(val - maxv);
        pr[i] = e;
        sum += e;
    }
    for (int64_t i = 0; i < K; ++i) pr[i] /= sum;
    int64_t cut = K;
    float cum = 0.0f;
    for (int64_t i = 0; i < K; ++i) {
        cum += pr[i];
        if (cum >= top_p) { cut = i + 1; break; }
    }
    float sub = 0.0f;
    for (int64_t i = 0; i < cut; ++i) sub += pr[i];
    for (int64_t i = 0; i < cut; ++i) pr[i] /= sub;
    float cdf = 0.0f;
    int64_t sel = cut - 1;
    for (int64_t i = 0; i < cut; ++i) {
        cdf += pr[i];
        if (u <= cdf) { sel = i; break; }
    }
    int64_t out = idx[sel];
    free(lg); free(idx); free(pr);
    return out;
}
