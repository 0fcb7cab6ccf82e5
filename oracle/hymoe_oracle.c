/* hymoe_oracle.c — CPU restatement of the reference MoE path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA path, never the product.
 * Built with -O2 -ffp-contract=off so every float operation is a separately rounded
 * IEEE mul or add in the same order as the reference; that makes the restatement
 * bit-identical to the compiled reference (oracle/_ref) on the same inputs.
 *
 * Reference anchors (paths within MaurerAnton/hunyuan-image-3-80b.cpp):
 *   router GEMV ......... src/attention.cpp:213-222
 *   softmax ............. src/attention.cpp:224-240
 *   top-8 + renorm ...... src/attention.cpp:242-276
 *   shared expert ....... src/attention.cpp:206-209
 *   routed loop ......... src/attention.cpp:282-300
 *   combine ............. src/attention.cpp:306-309
 *   residual (caller) ... src/decoder_layer.cpp:42
 *   SwiGLU FFN .......... src/rms_norm.cpp:39-91 (silu of the FIRST half, :70-74)
 *   RMSNorm ............. src/rms_norm.cpp:9-33
 *   GGUF Q4_0/Q8_0 ...... gguf-py 0.19.0 gguf/quants.py (Q4_0/Q8_0 quantize_blocks /
 *                         dequantize_blocks), the format the converter call sites
 *                         scripts/convert_to_gguf.py:200,245 name.  The reference
 *                         loader's own Q4_0 decoder (src/hunyuan_gguf_loader.cpp:41-72)
 *                         does not follow GGUF and is deliberately not restated.
 */
#define _GNU_SOURCE
#include "hymoe_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ threads */

typedef void (*range_fn)(void* arg, uint64_t lo, uint64_t hi);
typedef struct {
    range_fn fn;
    void* arg;
    uint64_t lo, hi;
} range_job;

static void* range_tramp(void* p) {
    range_job* j = (range_job*)p;
    j->fn(j->arg, j->lo, j->hi);
    return NULL;
}

/* Splits [0, n) into contiguous ranges, one per thread.  Results never depend on
 * the split: every output element is computed by exactly one sequential loop. */
static void parallel_for(uint64_t n, int nthreads, range_fn fn, void* arg) {
    if (nthreads < 1) nthreads = 1;
    if ((uint64_t)nthreads > n) nthreads = (int)(n ? n : 1);
    if (nthreads == 1) {
        fn(arg, 0, n);
        return;
    }
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * nthreads);
    range_job* jobs = (range_job*)malloc(sizeof(range_job) * nthreads);
    for (int t = 0; t < nthreads; ++t) {
        jobs[t].fn = fn;
        jobs[t].arg = arg;
        jobs[t].lo = n * (uint64_t)t / (uint64_t)nthreads;
        jobs[t].hi = n * (uint64_t)(t + 1) / (uint64_t)nthreads;
        pthread_create(&th[t], NULL, range_tramp, &jobs[t]);
    }
    for (int t = 0; t < nthreads; ++t) pthread_join(th[t], NULL);
    free(th);
    free(jobs);
}

/* ------------------------------------------------------------------ Philox */

void oracle_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
    uint32_t c0 = ctr[0], c1 = ctr[1], c2 = ctr[2], c3 = ctr[3];
    uint32_t k0 = key[0], k1 = key[1];
    for (int r = 0; r < 10; ++r) {
        if (r) {
            k0 += 0x9E3779B9u;
            k1 += 0xBB67AE85u;
        }
        const uint64_t p0 = (uint64_t)0xD2511F53u * c0;
        const uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
        const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
        const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
        c1 = (uint32_t)p1;
        c3 = (uint32_t)p0;
        c0 = n0;
        c2 = n2;
    }
    out[0] = c0;
    out[1] = c1;
    out[2] = c2;
    out[3] = c3;
}

float oracle_synth_scale(float stddev) {
    return (float)((double)stddev * sqrt(1.5) / 65536.0);
}

static inline float synth_value(uint64_t i, uint64_t seed, uint64_t stream, float c) {
    const uint32_t ctr[4] = {(uint32_t)i, (uint32_t)(i >> 32), (uint32_t)stream,
                             (uint32_t)(stream >> 32)};
    const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
    uint32_t r[4];
    oracle_philox4x32_10(ctr, key, r);
    int32_t s = 0;
    for (int w = 0; w < 4; ++w) s += (int32_t)(r[w] & 0xFFFFu) + (int32_t)(r[w] >> 16);
    return (float)(s - 262140) * c;
}

typedef struct {
    float* dst;
    uint64_t seed, stream;
    float c;
} fill_arg;

static void fill_range(void* p, uint64_t lo, uint64_t hi) {
    fill_arg* a = (fill_arg*)p;
    for (uint64_t i = lo; i < hi; ++i) a->dst[i] = synth_value(i, a->seed, a->stream, a->c);
}

void oracle_fill_normal(float* dst, uint64_t n, uint64_t seed, uint64_t stream, float stddev,
                        int nthreads) {
    fill_arg a = {dst, seed, stream, oracle_synth_scale(stddev)};
    parallel_for(n, nthreads, fill_range, &a);
}

/* ------------------------------------------------------------------ binary16 */

uint16_t oracle_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u);
    if (ax >= 0x477FF000u) return sign | 0x7C00u; /* >= 65520 rounds to infinity */
    const int e = (int)(ax >> 23);
    if (e < 113) { /* below 2^-14: binary16 subnormal, unit 2^-24 */
        const int shift = 126 - e;
        if (shift > 24) return sign;
        const uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
        uint32_t q = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        return sign | (uint16_t)q;
    }
    uint32_t h = ((uint32_t)(e - 112) << 10) | ((ax >> 13) & 0x3FFu);
    const uint32_t rem = ax & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return sign | (uint16_t)h;
}

float oracle_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else { /* subnormal: value m * 2^-24, exact in binary32 */
            float v = (float)m * 5.9604644775390625e-08f;
            memcpy(&bits, &v, 4);
            bits |= sign;
        }
    } else if (e == 31) {
        bits = sign | 0x7F800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* ------------------------------------------------------------------ GGUF blocks */

uint64_t oracle_type_nbytes(int type, uint64_t n) {
    switch (type) {
        case ORACLE_F32: return n * 4;
        case ORACLE_F16: return n * 2;
        case ORACLE_Q4_0: return n / 32 * 18;
        case ORACLE_Q8_0: return n / 32 * 34;
        default: return 0;
    }
}

static void put_f16(uint8_t* p, float f) {
    const uint16_t h = oracle_f32_to_f16(f);
    p[0] = (uint8_t)h;
    p[1] = (uint8_t)(h >> 8);
}

static float get_f16(const uint8_t* p) { return oracle_f16_to_f32((uint16_t)(p[0] | (p[1] << 8))); }

/* gguf/quants.py Q4_0.quantize_blocks: d = (value of largest magnitude, first on ties)
 * / -8; q = min(15, trunc(x/d + 8.5)). */
static void quant_q4_0_block(const float* x, uint8_t* b) {
    float amax = 0.0f, vmax = 0.0f;
    for (int j = 0; j < 32; ++j) {
        const float a = fabsf(x[j]);
        if (a > amax) {
            amax = a;
            vmax = x[j];
        }
    }
    const float d = vmax / -8.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    uint8_t q[32];
    for (int j = 0; j < 32; ++j) {
        const float t = truncf(x[j] * id + 8.5f);
        int v = t < 0.0f ? 0 : (int)t;
        q[j] = (uint8_t)(v > 15 ? 15 : v);
    }
    put_f16(b, d);
    for (int j = 0; j < 16; ++j) b[2 + j] = (uint8_t)(q[j] | (q[j + 16] << 4));
}

/* gguf/quants.py Q8_0.quantize_blocks: d = max|x| / 127; q = round-half-away(x/d). */
static void quant_q8_0_block(const float* x, uint8_t* b) {
    float amax = 0.0f;
    for (int j = 0; j < 32; ++j) {
        const float a = fabsf(x[j]);
        if (a > amax) amax = a;
    }
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    put_f16(b, d);
    for (int j = 0; j < 32; ++j) b[2 + j] = (uint8_t)(int8_t)roundf(x[j] * id);
}

void oracle_quantize(int type, const float* x, uint8_t* dst, uint64_t n) {
    switch (type) {
        case ORACLE_F32: memcpy(dst, x, n * 4); break;
        case ORACLE_F16:
            for (uint64_t i = 0; i < n; ++i) put_f16(dst + 2 * i, x[i]);
            break;
        case ORACLE_Q4_0:
            for (uint64_t b = 0; b < n / 32; ++b) quant_q4_0_block(x + 32 * b, dst + 18 * b);
            break;
        case ORACLE_Q8_0:
            for (uint64_t b = 0; b < n / 32; ++b) quant_q8_0_block(x + 32 * b, dst + 34 * b);
            break;
        default: break;
    }
}

void oracle_dequantize(int type, const uint8_t* src, float* dst, uint64_t n) {
    switch (type) {
        case ORACLE_F32: memcpy(dst, src, n * 4); break;
        case ORACLE_F16:
            for (uint64_t i = 0; i < n; ++i) dst[i] = get_f16(src + 2 * i);
            break;
        case ORACLE_Q4_0:
            for (uint64_t b = 0; b < n / 32; ++b) {
                const uint8_t* p = src + 18 * b;
                const float d = get_f16(p);
                for (int j = 0; j < 16; ++j) {
                    dst[32 * b + j] = (float)((int)(p[2 + j] & 0xF) - 8) * d;
                    dst[32 * b + j + 16] = (float)((int)(p[2 + j] >> 4) - 8) * d;
                }
            }
            break;
        case ORACLE_Q8_0:
            for (uint64_t b = 0; b < n / 32; ++b) {
                const uint8_t* p = src + 34 * b;
                const float d = get_f16(p);
                for (int j = 0; j < 32; ++j) dst[32 * b + j] = (float)(int8_t)p[2 + j] * d;
            }
            break;
        default: break;
    }
}

typedef struct {
    int type;
    uint8_t* qdst;
    float* fdst;
    uint64_t seed, stream;
    float c;
} synth_arg;

/* Works on 32-element blocks so a thread range never splits a GGUF block. */
static void synth_range(void* p, uint64_t blo, uint64_t bhi) {
    synth_arg* a = (synth_arg*)p;
    float x[32];
    uint8_t q[128]; /* one block of the widest type (F32: 128 bytes) */
    const uint64_t bb = oracle_type_nbytes(a->type, 32);
    for (uint64_t b = blo; b < bhi; ++b) {
        for (int j = 0; j < 32; ++j) x[j] = synth_value(32 * b + j, a->seed, a->stream, a->c);
        if (a->type == ORACLE_F32) {
            if (a->qdst) memcpy(a->qdst + bb * b, x, 128);
            if (a->fdst) memcpy(a->fdst + 32 * b, x, 128);
            continue;
        }
        uint8_t* qb = a->qdst ? a->qdst + bb * b : q;
        oracle_quantize(a->type, x, qb, 32);
        if (a->fdst) oracle_dequantize(a->type, qb, a->fdst + 32 * b, 32);
    }
}

void oracle_synth_tensor(int type, uint8_t* dst, uint64_t n, uint64_t seed, uint64_t stream,
                         float stddev, int nthreads) {
    synth_arg a = {type, dst, NULL, seed, stream, oracle_synth_scale(stddev)};
    parallel_for(n / 32, nthreads, synth_range, &a);
}

void oracle_synth_tensor_f32(int type, float* dst, uint64_t n, uint64_t seed, uint64_t stream,
                             float stddev, int nthreads) {
    synth_arg a = {type, NULL, dst, seed, stream, oracle_synth_scale(stddev)};
    parallel_for(n / 32, nthreads, synth_range, &a);
}

/* ------------------------------------------------------------------ RMSNorm */

void oracle_rms_norm(const float* x, const float* weight, float* out, uint32_t T, uint32_t H,
                     float eps) {
    for (uint32_t t = 0; t < T; ++t) {
        const float* row = x + (size_t)t * H;
        float ss = 0.0f;
        for (uint32_t j = 0; j < H; ++j) ss += row[j] * row[j];
        const float inv = 1.0f / sqrtf(ss / (float)H + eps);
        for (uint32_t j = 0; j < H; ++j) out[(size_t)t * H + j] = row[j] * inv * weight[j];
    }
}

/* ------------------------------------------------------------------ SwiGLU FFN */

/* One row through the FFN.  `mid` is scratch of 3*I floats. */
static void ffn_row(const float* x, const float* gu, const float* dn, float* y, uint32_t H,
                    uint32_t I, float* mid) {
    float* proj = mid;         /* [2I]: gate || up */
    float* act = mid + 2 * I;  /* [I] */
    for (uint32_t r = 0; r < 2 * I; ++r) {
        const float* w = gu + (size_t)r * H;
        float acc = 0.0f;
        for (uint32_t k = 0; k < H; ++k) acc += x[k] * w[k];
        proj[r] = acc;
    }
    for (uint32_t j = 0; j < I; ++j) {
        const float g = proj[j];
        const float sig = 1.0f / (1.0f + expf(-g));
        const float sg = g * sig;
        act[j] = sg * proj[I + j];
    }
    for (uint32_t r = 0; r < H; ++r) {
        const float* w = dn + (size_t)r * I;
        float acc = 0.0f;
        for (uint32_t k = 0; k < I; ++k) acc += act[k] * w[k];
        y[r] = acc;
    }
}

typedef struct {
    const float *x, *gu, *dn;
    float* out;
    uint32_t H, I;
} ffn_arg;

static void ffn_range(void* p, uint64_t lo, uint64_t hi) {
    ffn_arg* a = (ffn_arg*)p;
    float* mid = (float*)malloc(sizeof(float) * 3 * a->I);
    for (uint64_t t = lo; t < hi; ++t)
        ffn_row(a->x + t * a->H, a->gu, a->dn, a->out + t * a->H, a->H, a->I, mid);
    free(mid);
}

void oracle_swiglu_ffn(const float* x, const float* gate_up, const float* down, float* out,
                       uint32_t n, uint32_t H, uint32_t I, int nthreads) {
    ffn_arg a = {x, gate_up, down, out, H, I};
    parallel_for(n, nthreads, ffn_range, &a);
}

/* ------------------------------------------------------------------ router */

typedef struct {
    const float *x, *rw, *bias;
    uint32_t H, E, K;
    float *logits, *probs, *tw;
    int32_t* ti;
} router_arg;

static void router_token(const router_arg* a, uint64_t t, float* lg, float* pr) {
    const float* xr = a->x + t * a->H;
    for (uint32_t e = 0; e < a->E; ++e) {
        const float* w = a->rw + (size_t)e * a->H;
        float acc = 0.0f;
        for (uint32_t k = 0; k < a->H; ++k) acc += xr[k] * w[k];
        lg[e] = a->bias ? acc + a->bias[e] : acc;
    }
    float mx = lg[0];
    for (uint32_t e = 1; e < a->E; ++e)
        if (lg[e] > mx) mx = lg[e];
    float tot = 0.0f;
    for (uint32_t e = 0; e < a->E; ++e) {
        pr[e] = expf(lg[e] - mx);
        tot += pr[e];
    }
    for (uint32_t e = 0; e < a->E; ++e) pr[e] /= tot;
    /* Top-K by repeated selection: largest probability first, the lower expert index
     * first among equal probabilities (the order the reference's insertion with a
     * strict '<' produces). */
    uint64_t taken[4] = {0, 0, 0, 0};
    float sel_p[64];
    int32_t sel_e[64];
    for (uint32_t k = 0; k < a->K; ++k) {
        int32_t best = -1;
        for (uint32_t e = 0; e < a->E; ++e) {
            if (taken[e >> 6] >> (e & 63) & 1u) continue;
            if (best < 0 || pr[e] > pr[best]) best = (int32_t)e;
        }
        taken[best >> 6] |= 1ull << (best & 63);
        sel_p[k] = pr[best];
        sel_e[k] = best;
    }
    float s = 0.0f;
    for (uint32_t k = 0; k < a->K; ++k) s += sel_p[k];
    for (uint32_t k = 0; k < a->K; ++k) {
        if (a->tw) a->tw[t * a->K + k] = sel_p[k] / s;
        if (a->ti) a->ti[t * a->K + k] = sel_e[k];
    }
}

static void router_range(void* p, uint64_t lo, uint64_t hi) {
    router_arg* a = (router_arg*)p;
    float lg[256], pr[256];
    for (uint64_t t = lo; t < hi; ++t) {
        router_token(a, t, lg, pr);
        if (a->logits) memcpy(a->logits + t * a->E, lg, sizeof(float) * a->E);
        if (a->probs) memcpy(a->probs + t * a->E, pr, sizeof(float) * a->E);
    }
}

void oracle_router(const float* x, uint32_t T, uint32_t H, uint32_t E, uint32_t K,
                   const float* router_w, const float* bias, float* logits, float* probs,
                   float* topk_w, int32_t* topk_idx, int nthreads) {
    router_arg a = {x, router_w, bias, H, E, K, logits, probs, topk_w, topk_idx};
    parallel_for(T, nthreads, router_range, &a);
}

/* ------------------------------------------------------------------ MoE block */

typedef struct {
    const float *x, *resid, *sgu, *sdn;
    const float *const *egu, *const *edn;
    const float* tw;
    const int32_t* ti;
    float* out;
    uint32_t H, I, K;
} moe_arg;

static void moe_range(void* p, uint64_t lo, uint64_t hi) {
    moe_arg* a = (moe_arg*)p;
    const uint32_t H = a->H;
    float* mid = (float*)malloc(sizeof(float) * 3 * a->I);
    float* shared = (float*)malloc(sizeof(float) * H);
    float* routed = (float*)malloc(sizeof(float) * H);
    float* y = (float*)malloc(sizeof(float) * H);
    for (uint64_t t = lo; t < hi; ++t) {
        const float* xr = a->x + t * H;
        ffn_row(xr, a->sgu, a->sdn, shared, H, a->I, mid);
        for (uint32_t j = 0; j < H; ++j) routed[j] = 0.0f;
        for (uint32_t k = 0; k < a->K; ++k) {
            const int32_t e = a->ti[t * a->K + k];
            const float wk = a->tw[t * a->K + k];
            ffn_row(xr, a->egu[e], a->edn[e], y, H, a->I, mid);
            for (uint32_t j = 0; j < H; ++j) routed[j] += wk * y[j];
        }
        float* o = a->out + t * H;
        for (uint32_t j = 0; j < H; ++j) {
            const float m = shared[j] + routed[j];
            o[j] = a->resid ? a->resid[t * H + j] + m : m;
        }
    }
    free(mid);
    free(shared);
    free(routed);
    free(y);
}

int oracle_moe_forward(const float* x, const float* resid, uint32_t T, uint32_t H, uint32_t I,
                       uint32_t E, uint32_t K, const float* router_w, const float* bias,
                       const float* shared_gu, const float* shared_down,
                       const float* const* experts_gu, const float* const* experts_down,
                       float* out, float* dbg_logits, float* dbg_probs, float* dbg_w,
                       int32_t* dbg_idx, int nthreads) {
    if (E > 256 || K > E || K > 64) return -1;
    float* tw = (float*)malloc(sizeof(float) * (size_t)T * K);
    int32_t* ti = (int32_t*)malloc(sizeof(int32_t) * (size_t)T * K);
    oracle_router(x, T, H, E, K, router_w, bias, dbg_logits, dbg_probs, tw, ti, nthreads);
    int rc = 0;
    for (uint64_t i = 0; i < (uint64_t)T * K; ++i)
        if (!experts_gu[ti[i]] || !experts_down[ti[i]]) rc = -1;
    if (rc == 0) {
        moe_arg a = {x, resid, shared_gu, shared_down, experts_gu, experts_down,
                     tw, ti, out, H, I, K};
        parallel_for(T, nthreads, moe_range, &a);
    }
    if (dbg_w) memcpy(dbg_w, tw, sizeof(float) * (size_t)T * K);
    if (dbg_idx) memcpy(dbg_idx, ti, sizeof(int32_t) * (size_t)T * K);
    free(tw);
    free(ti);
    return rc;
}


/* ------------------------------------------------------------------ FULL-mode routing */

/* softmax_f32 of src/hunyuan_moe_full.cpp:41-50: running max (strict >), expf of the
 * differences summed in order, each divided by the sum. */
static void full_softmax(float* x, uint32_t n) {
    float mx = x[0];
    for (uint32_t i = 1; i < n; ++i)
        if (x[i] > mx) mx = x[i];
    float sum = 0.0f;
    for (uint32_t i = 0; i < n; ++i) {
        x[i] = expf(x[i] - mx);
        sum += x[i];
    }
    for (uint32_t i = 0; i < n; ++i) x[i] /= sum;
}

/* The k largest of x[0..n) in decreasing order, equal values in increasing index order
 * (what the insertion of src/hunyuan_moe_full.cpp:56-82 keeps); slots past n are (0, 0). */
static void full_topk(const float* x, uint32_t n, uint32_t k, float* vals, int32_t* ids) {
    uint8_t taken[256] = {0};
    for (uint32_t r = 0; r < k; ++r) {
        int32_t b = -1;
        for (uint32_t i = 0; i < n && i < 256; ++i)
            if (!taken[i] && (b < 0 || x[i] > x[b])) b = (int32_t)i;
        if (b < 0) {
            vals[r] = 0.0f;
            ids[r] = 0;
            continue;
        }
        taken[b] = 1;
        vals[r] = x[b];
        ids[r] = b;
    }
}

void oracle_topkgating_full(const float* logits, uint32_t T, uint32_t E, uint32_t K,
                            int group_limited, uint32_t n_group, uint32_t topk_group,
                            int drop_tokens, float capacity_factor, uint32_t min_capacity,
                            int norm_topk_prob, float routed_scaling_factor, float* probs,
                            int32_t* idx, float* w, uint8_t* keep, int32_t* exp_counts,
                            uint32_t* capacity) {
    *capacity = 0;
    if (E == 0 || E > 256 || n_group > 256 || K == 0) return; /* the fixed tables below */
    const uint32_t nk = K > topk_group ? K : topk_group;    /* entries full_topk writes */
    float* gates = (float*)malloc(sizeof(float) * (size_t)T * E);
    float* tv = (float*)malloc(sizeof(float) * nk);
    int32_t* ti = (int32_t*)malloc(sizeof(int32_t) * nk);
    for (uint32_t t = 0; t < T; ++t) {
        float* g = gates + (size_t)t * E;
        memcpy(g, logits + (size_t)t * E, sizeof(float) * E);
        full_softmax(g, E);
        memcpy(probs + (size_t)t * E, g, sizeof(float) * E);
        if (group_limited && n_group > 0 && topk_group > 0) {
            const uint32_t gs = E / n_group;
            float score[256];
            for (uint32_t q = 0; q < n_group; ++q) {
                float m = 0.0f;
                for (uint32_t e = 0; e < gs; ++e)
                    if (g[q * gs + e] > m) m = g[q * gs + e];
                score[q] = m;
            }
            full_topk(score, n_group, topk_group, tv, ti);
            for (uint32_t q = 0; q < n_group; ++q) {
                int sel = 0;
                for (uint32_t r = 0; r < topk_group; ++r) sel |= ti[r] == (int32_t)q;
                if (!sel)
                    for (uint32_t e = 0; e < gs; ++e) g[q * gs + e] = 0.0f;
            }
        }
        full_topk(g, E, K, tv, idx + (size_t)t * K);
    }
    for (uint32_t e = 0; e < E; ++e) exp_counts[e] = 0;
    for (uint32_t i = 0; i < T * K; ++i) exp_counts[idx[i]]++;
    uint32_t cap;
    if (drop_tokens) {
        const uint32_t f = (uint32_t)(capacity_factor * (float)K * (float)T / (float)E);
        cap = f > K ? f : K;
    } else {
        cap = 0;
        for (uint32_t e = 0; e < E; ++e)
            if ((uint32_t)exp_counts[e] > cap) cap = (uint32_t)exp_counts[e];
    }
    if (cap < min_capacity) cap = min_capacity;
    *capacity = cap;
    for (uint32_t t = 0; t < T; ++t) {
        const float* g = gates + (size_t)t * E;
        const int32_t* id = idx + (size_t)t * K;
        if (norm_topk_prob && K > 1) {
            float s = 0.0f;
            for (uint32_t k = 0; k < K; ++k) s += g[id[k]];
            if (s < 1e-8f) s = 1e-8f;
            for (uint32_t k = 0; k < K; ++k) w[(size_t)t * K + k] = g[id[k]] / s;
        } else {
            for (uint32_t k = 0; k < K; ++k) w[(size_t)t * K + k] = g[id[k]] * routed_scaling_factor;
        }
    }
    /* priorities in k-major order */
    int32_t* seen = (int32_t*)calloc(E, sizeof(int32_t));
    for (uint32_t k = 0; k < K; ++k)
        for (uint32_t t = 0; t < T; ++t) {
            const int32_t e = idx[(size_t)t * K + k];
            keep[(size_t)t * K + k] = (uint32_t)seen[e] < cap;
            seen[e]++;
        }
    free(seen);
    free(gates);
    free(tv);
    free(ti);
}

