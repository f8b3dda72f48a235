/*
 * CPU oracle for the candle-moe hot path.  TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, what the reference crate kozistr/candle-moe computes on its
 * hot path, so that the CUDA product can be checked against it.  Only tests/, the smoke check in
 * __graft_entry__.py and bench.py's CPU-baseline leg may load it; the product library never links
 * or calls it.
 *
 * Parity pin: the reference ships no golden vectors (its tests draw unseeded device randn).  The
 * restatement is pinned against outputs of the reference's own CUDA kernels, built from the
 * reference sources by oracle/build_ref.sh and run on a B200; the fixtures live in tests/golden/
 * together with the script that produced them.
 *
 * Functions and the reference code each one follows:
 *   oracle_topk_softmax   kernels/topk_softmax.cu:136-266 (topkGatingSoftmax) and the launcher
 *                         constants at :268-295; the thread grouping of the row is reproduced so
 *                         that the float summation order of the softmax denominator matches.
 *   oracle_route_prep     kernels/preprocessing.cuh:5-59 (moe_preprocess_kernel): histogram,
 *                         exclusive scan, [E]=total, [E+1]=max count, scatter.  The reference's
 *                         within-expert order comes from atomics and is not deterministic; here it
 *                         is pinned to ascending flat index (token*k + slot).
 *   oracle_moe_forward    tests/moe_tests.rs:124-189 (naive per-expert loop) for the structure,
 *                         kernels/common.cuh:116-138 for the activations, kernels/moe.cu:193-449
 *                         for the f32 data flow, and nomic_moe.cu:374 / qwen3_moe.cu:493 /
 *                         qwen3_moe.cu:637-641 for where the f16/bf16 path rounds (intermediate and
 *                         each weighted contribution).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------------------------------ */
/* element conversion                                                                          */
/* ------------------------------------------------------------------------------------------ */

enum { DT_F16 = 0, DT_BF16 = 1, DT_F32 = 2 };

static inline float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline uint16_t f32_to_bf16_rne(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40); /* quiet NaN */
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}

static inline float f16_to_f32(uint16_t h) {
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float)v;
}

static inline uint16_t f32_to_f16_rne(float f) {
    _Float16 v = (_Float16)f;
    uint16_t h;
    memcpy(&h, &v, 2);
    return h;
}

static inline float round_to(float v, int dtype) {
    if (dtype == DT_BF16) return bf16_to_f32(f32_to_bf16_rne(v));
    if (dtype == DT_F16) return f16_to_f32(f32_to_f16_rne(v));
    return v;
}

static inline float load_elem(const void* p, size_t i, int dtype) {
    if (dtype == DT_F32) return ((const float*)p)[i];
    if (dtype == DT_BF16) return bf16_to_f32(((const uint16_t*)p)[i]);
    return f16_to_f32(((const uint16_t*)p)[i]);
}

EXPORT void oracle_convert_to_f32(const void* src, int dtype, size_t n, float* dst) {
    for (size_t i = 0; i < n; ++i) dst[i] = load_elem(src, i, dtype);
}

EXPORT void oracle_convert_from_f32(const float* src, int dtype, size_t n, void* dst) {
    for (size_t i = 0; i < n; ++i) {
        if (dtype == DT_F32) ((float*)dst)[i] = src[i];
        else if (dtype == DT_BF16) ((uint16_t*)dst)[i] = f32_to_bf16_rne(src[i]);
        else ((uint16_t*)dst)[i] = f32_to_f16_rne(src[i]);
    }
}

/* ------------------------------------------------------------------------------------------ */
/* seeded RNG: SplitMix64 + Box-Muller (the synthetic-input generator of the benches/tests)     */
/* ------------------------------------------------------------------------------------------ */

static inline uint64_t splitmix64(uint64_t* s) {
    uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* n normal deviates N(mean, std) written as `dtype`; stream `seed` is split into fixed blocks of
 * 4096 values so that the output does not depend on the thread count. */
EXPORT void oracle_randn(uint64_t seed, size_t n, float mean, float stdv, int dtype, void* dst,
                         int nthreads) {
    const size_t BLK = 4096;
    size_t nblk = (n + BLK - 1) / BLK;
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(static)
#endif
    for (size_t b = 0; b < nblk; ++b) {
        uint64_t s = seed * 0x2545F4914F6CDD1Dull + b * 0x9E3779B97F4A7C15ull + 1;
        splitmix64(&s);
        size_t lo = b * BLK, hi = lo + BLK < n ? lo + BLK : n;
        for (size_t i = lo; i < hi; i += 2) {
            double u1 = ((splitmix64(&s) >> 11) + 1.0) * (1.0 / 9007199254740993.0);
            double u2 = (splitmix64(&s) >> 11) * (1.0 / 9007199254740992.0);
            double r = sqrt(-2.0 * log(u1));
            double z0 = r * cos(6.283185307179586 * u2), z1 = r * sin(6.283185307179586 * u2);
            float v0 = (float)(mean + stdv * z0), v1 = (float)(mean + stdv * z1);
            if (dtype == DT_F32) {
                ((float*)dst)[i] = v0;
                if (i + 1 < hi) ((float*)dst)[i + 1] = v1;
            } else if (dtype == DT_BF16) {
                ((uint16_t*)dst)[i] = f32_to_bf16_rne(v0);
                if (i + 1 < hi) ((uint16_t*)dst)[i + 1] = f32_to_bf16_rne(v1);
            } else {
                ((uint16_t*)dst)[i] = f32_to_f16_rne(v0);
                if (i + 1 < hi) ((uint16_t*)dst)[i + 1] = f32_to_f16_rne(v1);
            }
        }
    }
}

/* ------------------------------------------------------------------------------------------ */
/* router: kernels/topk_softmax.cu:136-266                                                      */
/* ------------------------------------------------------------------------------------------ */

/* Thread grouping of one row in the reference launcher (topk_softmax.cu:268-295):
 * BYTES_PER_LDG = min(16, 4E); ELTS_PER_LDG = BYTES_PER_LDG/4; VPT = max(1, E/(ELTS*32))*ELTS;
 * THREADS_PER_ROW = E/VPT.  Thread g of the row holds columns g*ELTS + l*ELTS*TPR + i. */
static void router_geometry(int E, int* elts, int* vpt, int* tpr) {
    int bytes = 4 * E < 16 ? 4 * E : 16;
    int el = bytes / 4;
    int vecs = E / (el * 32);
    if (vecs < 1) vecs = 1;
    *elts = el;
    *vpt = vecs * el;
    *tpr = E / *vpt;
}

/*
 * logits [T,E] f32 -> weights [T,k] f32, indices [T,k] i32, src [T,k] i32 (= j*T + t).
 * near_tie (optional, [T] u8): set to 1 when any pick of the row was decided between unequal values
 * that are within 8 ulps of each other; on such rows a GPU using a different exp() may legitimately
 * choose differently.  renorm != 0 divides the k weights by their sum (Qwen3 norm_topk_prob; the
 * reference itself never renormalises).
 */
EXPORT void oracle_topk_softmax(const float* logits, int T, int E, int k, int renorm,
                                float* weights, int32_t* indices, int32_t* src, uint8_t* near_tie) {
    int elts, vpt, tpr;
    router_geometry(E, &elts, &vpt, &tpr);
    int ldgs = vpt / elts;
    float* p = (float*)malloc(sizeof(float) * (size_t)E);
    float* part = (float*)malloc(sizeof(float) * (size_t)tpr);
    float* nxt = (float*)malloc(sizeof(float) * (size_t)tpr);
    for (int t = 0; t < T; ++t) {
        const float* row = logits + (size_t)t * E;
        float m = row[0];
        for (int c = 1; c < E; ++c) m = fmaxf(m, row[c]);
        /* per-thread partial sums in the thread's own element order */
        for (int g = 0; g < tpr; ++g) {
            float s = 0.f;
            for (int l = 0; l < ldgs; ++l)
                for (int i = 0; i < elts; ++i) {
                    int c = g * elts + l * elts * tpr + i;
                    float e = expf(row[c] - m);
                    p[c] = e;
                    s += e;
                }
            part[g] = s;
        }
        for (int mask = tpr / 2; mask > 0; mask /= 2) {
            for (int g = 0; g < tpr; ++g) nxt[g] = part[g] + part[g ^ mask];
            memcpy(part, nxt, sizeof(float) * (size_t)tpr);
        }
        float recip = 1.f / part[0];
        for (int c = 0; c < E; ++c) p[c] = p[c] * recip;
        uint8_t tie = 0;
        float wsum = 0.f;
        for (int j = 0; j < k; ++j) {
            /* global argmax, ties -> lowest expert (topk_softmax.cu:220-248) */
            int best = 0;
            for (int c = 1; c < E; ++c)
                if (p[c] > p[best]) best = c;
            float bv = p[best];
            float second = -INFINITY;
            for (int c = 0; c < E; ++c)
                if (c != best && p[c] > second) second = p[c];
            /* exact ties resolve the same way everywhere (equal inputs give equal exp());
             * only near-but-unequal values can flip under a different exp() */
            if (E > 1 && bv != second && bv - second <= 8.f * ldexpf(1.f, ilogbf(fabsf(bv) + 1e-30f) - 23)) tie = 1;
            weights[(size_t)t * k + j] = bv;
            indices[(size_t)t * k + j] = best;
            src[(size_t)t * k + j] = j * T + t;
            wsum += bv;
            p[best] = -10000.f; /* topk_softmax.cu:256-264 */
        }
        if (renorm) {
            for (int j = 0; j < k; ++j) weights[(size_t)t * k + j] /= wsum;
        }
        if (near_tie) near_tie[t] = tie;
    }
    free(p);
    free(part);
    free(nxt);
}

/* ------------------------------------------------------------------------------------------ */
/* route preparation: kernels/preprocessing.cuh:5-59                                            */
/* ------------------------------------------------------------------------------------------ */

/*
 * indices [T*k] (u32 bit patterns, ids >= E are skipped, preprocessing.cuh:29), weights [T*k] f32.
 * offsets [E+2]: exclusive prefix of per-expert counts, offsets[E] = routed rows, offsets[E+1] =
 * max count.  sorted_token [rows] = token id, sorted_weight [rows], sorted_flat [rows] = t*k+j;
 * within an expert rows are in ascending flat index.
 */
EXPORT void oracle_route_prep(const uint32_t* indices, const float* weights, int T, int k, int E,
                              int32_t* offsets, int32_t* sorted_token, float* sorted_weight,
                              int32_t* sorted_flat) {
    int64_t total = (int64_t)T * k;
    int32_t* cursor = (int32_t*)calloc((size_t)E + 1, sizeof(int32_t));
    for (int64_t i = 0; i < total; ++i) {
        uint32_t e = indices[i];
        if (e < (uint32_t)E) cursor[e]++;
    }
    int32_t sum = 0, mx = 0;
    for (int e = 0; e < E; ++e) {
        int32_t c = cursor[e];
        offsets[e] = sum;
        if (c > mx) mx = c;
        cursor[e] = sum;
        sum += c;
    }
    offsets[E] = sum;
    offsets[E + 1] = mx;
    for (int64_t i = 0; i < total; ++i) {
        uint32_t e = indices[i];
        if (e >= (uint32_t)E) continue;
        int32_t pos = cursor[e]++;
        if (sorted_token) sorted_token[pos] = (int32_t)(i / k);
        if (sorted_weight) sorted_weight[pos] = weights[i];
        if (sorted_flat) sorted_flat[pos] = (int32_t)i;
    }
    free(cursor);
}

/* ------------------------------------------------------------------------------------------ */
/* activations: kernels/common.cuh:116-138                                                      */
/* ------------------------------------------------------------------------------------------ */

static inline float act_f32(float x, int act) {
    switch (act) {
        case 1: {
            const float c0 = 0.7978845608f, c1 = 0.044715f;
            float x3 = x * x * x;
            return 0.5f * x * (1.0f + tanhf(c0 * (x + c1 * x3)));
        }
        case 2: return fmaxf(0.0f, x);
        default: return x / (1.0f + expf(-x)); /* 0 and unknown ids: SiLU (common.cuh:136) */
    }
}

EXPORT float oracle_activation(float x, int act) { return act_f32(x, act); }

/* ------------------------------------------------------------------------------------------ */
/* fused MoE forward: tests/moe_tests.rs:124-189 + kernels/moe.cu:193-449                       */
/* ------------------------------------------------------------------------------------------ */

#define ROW_BLOCK 8

/*
 * x [T,H], gate/up [E,H,I], down [E,I,H] (Qwen3, moe_type 0) or NULL (Nomic, moe_type 1),
 * all of element type `dtype` (0 f16, 1 bf16, 2 f32); routing weights [T,k] f32; indices [T,k]
 * u32.  out [T,H] f32 receives the f32 value before the final rounding to `dtype`.
 *
 * Qwen3: h = act(x.G_e) * (x.U_e);  y = h.D_e        (qwen3_moe.cu:492, 637-641)
 * Nomic: h = act(x.G_e);            y = h.U_e^T      (nomic_moe.cu:645, 463)
 * out[t] = sum over slots j (in slot order) of w[t,j] * y_{e(t,j)}(t), accumulated in f32.
 *
 * round_dtype (0 f16 / 1 bf16 / 2 none) rounds the intermediate h and each weighted contribution
 * to that type, as the reference's f16/bf16 GEMM path does (nomic_moe.cu:374, qwen3_moe.cu:493,
 * qwen3_moe.cu:637-641).  All products accumulate in f32.
 */
/* max_contrib (may be NULL): [T,H] largest |weighted contribution| among each token's slots,
 * after rounding -- the scale of the rounding steps the result is built from, which the tests use
 * to tell a one-unit rounding disagreement in a contribution from a wrong result. */
EXPORT int oracle_moe_forward_ex(const void* x, const void* gate, const void* up, const void* down,
                                 const float* routing_w, const uint32_t* indices, int T, int H,
                                 int I, int E, int k, int act, int moe_type, int dtype,
                                 int round_dtype, int nthreads, float* out, float* max_contrib) {
    int64_t rows = (int64_t)T * k;
    int32_t* offsets = (int32_t*)malloc(sizeof(int32_t) * ((size_t)E + 2));
    int32_t* sflat = (int32_t*)malloc(sizeof(int32_t) * (size_t)(rows > 0 ? rows : 1));
    float* sw = (float*)malloc(sizeof(float) * (size_t)(rows > 0 ? rows : 1));
    float* contrib = (float*)calloc((size_t)(rows > 0 ? rows : 1) * (size_t)H, sizeof(float));
    if (!offsets || !sflat || !sw || !contrib) {
        free(offsets); free(sflat); free(sw); free(contrib);
        return -1;
    }
    oracle_route_prep(indices, routing_w, T, k, E, offsets, NULL, sw, sflat);

    /* work items: (expert, block of ROW_BLOCK rows) */
    int64_t nitems = 0;
    for (int e = 0; e < E; ++e) nitems += (offsets[e + 1] - offsets[e] + ROW_BLOCK - 1) / ROW_BLOCK;
    int64_t* item_e = (int64_t*)malloc(sizeof(int64_t) * (size_t)(nitems > 0 ? nitems : 1));
    int64_t* item_r = (int64_t*)malloc(sizeof(int64_t) * (size_t)(nitems > 0 ? nitems : 1));
    {
        int64_t n = 0;
        for (int e = 0; e < E; ++e) {
            int32_t lo = offsets[e], hi = offsets[e + 1];
            for (int32_t r = lo; r < hi; r += ROW_BLOCK) { item_e[n] = e; item_r[n] = r; ++n; }
        }
    }
    const int qwen3 = (moe_type == 0);
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel
#endif
    {
        float* xa = (float*)malloc(sizeof(float) * ROW_BLOCK * (size_t)H);
        float* hg = (float*)malloc(sizeof(float) * ROW_BLOCK * (size_t)I);
        float* hu = (float*)malloc(sizeof(float) * ROW_BLOCK * (size_t)I);
        float* wrow = (float*)malloc(sizeof(float) * (size_t)(I > H ? I : H));
        float* y = (float*)malloc(sizeof(float) * ROW_BLOCK * (size_t)H);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int64_t it = 0; it < nitems; ++it) {
            int e = (int)item_e[it];
            int32_t r0 = (int32_t)item_r[it];
            int32_t rend = offsets[e + 1];
            int nr = rend - r0 < ROW_BLOCK ? rend - r0 : ROW_BLOCK;
            for (int r = 0; r < nr; ++r) {
                int64_t tok = sflat[r0 + r] / k;
                for (int h = 0; h < H; ++h) xa[(size_t)r * H + h] = load_elem(x, (size_t)tok * H + h, dtype);
            }
            memset(hg, 0, sizeof(float) * ROW_BLOCK * (size_t)I);
            memset(hu, 0, sizeof(float) * ROW_BLOCK * (size_t)I);
            size_t wbase = (size_t)e * H * I;
            /* GEMM-1: h[r,i] = sum_h x[r,h] * W[h,i]  (axpy over i, k-ascending) */
            for (int h = 0; h < H; ++h) {
                for (int i = 0; i < I; ++i) wrow[i] = load_elem(gate, wbase + (size_t)h * I + i, dtype);
                for (int r = 0; r < nr; ++r) {
                    float a = xa[(size_t)r * H + h];
                    float* dst = hg + (size_t)r * I;
                    for (int i = 0; i < I; ++i) dst[i] += a * wrow[i];
                }
                if (qwen3) {
                    for (int i = 0; i < I; ++i) wrow[i] = load_elem(up, wbase + (size_t)h * I + i, dtype);
                    for (int r = 0; r < nr; ++r) {
                        float a = xa[(size_t)r * H + h];
                        float* dst = hu + (size_t)r * I;
                        for (int i = 0; i < I; ++i) dst[i] += a * wrow[i];
                    }
                }
            }
            for (int r = 0; r < nr; ++r)
                for (int i = 0; i < I; ++i) {
                    size_t o = (size_t)r * I + i;
                    float v = act_f32(hg[o], act);
                    if (qwen3) v = v * hu[o];
                    hg[o] = (round_dtype == DT_F32) ? v : round_to(v, round_dtype);
                }
            memset(y, 0, sizeof(float) * ROW_BLOCK * (size_t)H);
            if (qwen3) {
                /* GEMM-2: y[r,n] = sum_i h[r,i] * D[i,n] */
                size_t dbase = (size_t)e * I * H;
                for (int i = 0; i < I; ++i) {
                    for (int n = 0; n < H; ++n) wrow[n] = load_elem(down, dbase + (size_t)i * H + n, dtype);
                    for (int r = 0; r < nr; ++r) {
                        float a = hg[(size_t)r * I + i];
                        float* dst = y + (size_t)r * H;
                        for (int n = 0; n < H; ++n) dst[n] += a * wrow[n];
                    }
                }
            } else {
                /* GEMM-2 (Nomic): y[r,n] = sum_i h[r,i] * U[n,i] */
                for (int n = 0; n < H; ++n) {
                    for (int i = 0; i < I; ++i) wrow[i] = load_elem(up, wbase + (size_t)n * I + i, dtype);
                    for (int r = 0; r < nr; ++r) {
                        const float* a = hg + (size_t)r * I;
                        float s = 0.f;
                        for (int i = 0; i < I; ++i) s += a[i] * wrow[i];
                        y[(size_t)r * H + n] = s;
                    }
                }
            }
            for (int r = 0; r < nr; ++r) {
                int64_t flat = sflat[r0 + r];
                float wgt = sw[r0 + r];
                float* dst = contrib + (size_t)flat * H;
                for (int n = 0; n < H; ++n) {
                    float v = y[(size_t)r * H + n] * wgt;
                    dst[n] = (round_dtype == DT_F32) ? v : round_to(v, round_dtype);
                }
            }
        }
        free(xa); free(hg); free(hu); free(wrow); free(y);
    }
    /* combine in slot order */
#ifdef _OPENMP
#pragma omp parallel for schedule(static)
#endif
    for (int64_t t = 0; t < T; ++t) {
        float* o = out + (size_t)t * H;
        for (int n = 0; n < H; ++n) o[n] = 0.f;
        for (int j = 0; j < k; ++j) {
            const float* c = contrib + ((size_t)t * k + j) * H;
            for (int n = 0; n < H; ++n) o[n] += c[n];
        }
        if (max_contrib) {
            float* mc = max_contrib + (size_t)t * H;
            for (int n = 0; n < H; ++n) mc[n] = 0.f;
            for (int j = 0; j < k; ++j) {
                const float* c = contrib + ((size_t)t * k + j) * H;
                for (int n = 0; n < H; ++n) mc[n] = fmaxf(mc[n], fabsf(c[n]));
            }
        }
    }
    free(item_e); free(item_r);
    free(offsets); free(sflat); free(sw); free(contrib);
    return 0;
}

EXPORT int oracle_moe_forward(const void* x, const void* gate, const void* up, const void* down,
                              const float* routing_w, const uint32_t* indices, int T, int H, int I,
                              int E, int k, int act, int moe_type, int dtype, int round_dtype,
                              int nthreads, float* out) {
    return oracle_moe_forward_ex(x, gate, up, down, routing_w, indices, T, H, I, E, k, act,
                                 moe_type, dtype, round_dtype, nthreads, out, NULL);
}

EXPORT int oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Threads the OpenMP loops above use from now on (n <= 0 leaves the setting unchanged); returns
 * the resulting count.  The CPU baselines set it to the host's core count explicitly, so that
 * an inherited OMP_NUM_THREADS (torchrun exports 1) does not shrink them. */
EXPORT int oracle_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
#else
    (void)n;
    return 1;
#endif
}
