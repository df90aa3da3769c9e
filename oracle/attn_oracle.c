/*
 * attn_oracle.c - CPU restatement of LiGGUF's attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA kernels: only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it.  The product library
 * (ligguf_b200/libligguf_cuda_attn.so) never calls into it and has no CPU fallback.
 *
 * What it restates (paths relative to the matrixsmaster/ligguf tree):
 *   - rope()            fast/lil_math.cpp:901-920, table fast/common.cpp:34,38-39
 *   - rmsnorm_inplace() fast/lil_math.cpp:931-937
 *   - softmax()         fast/lil_math.cpp:964-976 (two pass: max, exp+sum, divide)
 *   - fp32 -> fp16      fast/lil_math.cpp:57-76,83-86 (round to nearest even; NaN -> 0x7E00)
 *   - decode attention  fast/ligguf_fast_qk.cpp:42-105 (Qwen3 QK norm, RoPE, KV append, GQA
 *                       h/nrep mapping, scores, softmax, P.V; t == pos reads the fp32 k,v)
 *                       and its fp32-cache twin cpp/ligguf.cpp:674-718 /
 *                       cpp/ligguf_distrib.cpp:709-747 (scale by division)
 *   - prefill           = decode repeated for pos0..pos0+n-1, as feed_text() does
 *                       (fast/ligguf_fast_qk.cpp:340-356)
 *   - BERT attention    fast/vdb.cpp:189-212 (scores over all ntok tokens, softmax, P.V)
 *   - SARA shard map    cpp/ligguf_distrib.cpp:657-679 (split_even / build_shards)
 * plus the seeded synthetic generator that the CUDA library implements bit for bit
 * (ligguf_cuda_synth_fill in include/ligguf_cuda_attn.h).
 *
 * Arithmetic is plain IEEE fp32 (built with -ffp-contract=off), loops in the reference's order.
 * Parity of this restatement against the reference's own compiled code is checked by
 * tests/test_oracle.py against fixtures made by tests/golden/make_golden.py with
 * oracle/_ref/libligguf_ref.so (the reference's fast/lil_math.cpp built from source).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define LO_KV_F32 0
#define LO_KV_F16 1
#define LO_KV_BF16 2

/* ---------------------------------------------------------------- synthetic generator ---- */
uint64_t lo_splitmix64(uint64_t x)
{
    uint64_t z = x + 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

/* Standard deviation of the sum of four independent uniforms on {0..65535}. */
#define LO_SYNTH_SD 37837.227241611614

float lo_synth_mul(float scale) { return (float)((double)scale / LO_SYNTH_SD); }

static inline float lo_synth_one(uint64_t base, uint64_t idx, float mul, float add)
{
    const uint64_t r = lo_splitmix64(base + idx);
    const int32_t s = (int32_t)(r & 0xFFFF) + (int32_t)((r >> 16) & 0xFFFF) +
                      (int32_t)((r >> 32) & 0xFFFF) + (int32_t)(r >> 48) - 131070;
    const float prod = (float)s * mul; /* one rounding */
    return prod + add;                 /* one rounding (no contraction: -ffp-contract=off) */
}

uint64_t lo_synth_base(uint64_t seed, uint64_t stream)
{
    return lo_splitmix64(seed ^ (stream * 0xD1B54A32D192ED03ULL));
}

void lo_synth_fill_f32(float* dst, size_t n, uint64_t seed, uint64_t stream, uint64_t idx0,
                       float scale, float add)
{
    const uint64_t base = lo_synth_base(seed, stream);
    const float mul = lo_synth_mul(scale);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; i++) dst[i] = lo_synth_one(base, idx0 + (uint64_t)i, mul, add);
}

/* ---------------------------------------------------------------- half / bfloat16 ------- */
static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* IEEE binary16, round to nearest even; NaN becomes the quiet NaN 0x7E00 with the input sign,
 * the same encoding fast/lil_math.cpp:75 produces. */
uint16_t lo_f32_to_f16(float f)
{
    const uint32_t x = f2u(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7FFFFFFFu;
    if (ax > 0x7F800000u) return (uint16_t)(sign | 0x7E00u);
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* >= 65520 rounds to inf */
    if (ax < 0x38800000u) {                                  /* below 2^-14: subnormal half */
        if (ax < 0x33000000u) return (uint16_t)sign;         /* below 2^-25: zero */
        const uint32_t e = ax >> 23;
        const uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
        const uint32_t shift = 126u - e;                     /* units of 2^-24 */
        uint32_t q = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t h = (((ax >> 23) - 112u) << 10) | ((ax & 0x7FFFFFu) >> 13);
    const uint32_t rem = ax & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

float lo_f16_to_f32(uint16_t h)
{
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1Fu;
    const uint32_t m = h & 0x3FFu;
    if (e == 0) return u2f(sign | f2u((float)m * 5.9604644775390625e-8f)); /* m * 2^-24 */
    if (e == 31) return u2f(sign | 0x7F800000u | (m << 13));
    return u2f(sign | ((e + 112u) << 23) | (m << 13));
}

uint16_t lo_f32_to_bf16(float f)
{
    const uint32_t x = f2u(f);
    if ((x & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((x >> 16) | 0x40u);
    return (uint16_t)((x + 0x7FFFu + ((x >> 16) & 1u)) >> 16);
}

float lo_bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

static inline float kv_load(const void* base, int type, size_t i)
{
    if (type == LO_KV_F32) return ((const float*)base)[i];
    if (type == LO_KV_F16) return lo_f16_to_f32(((const uint16_t*)base)[i]);
    return lo_bf16_to_f32(((const uint16_t*)base)[i]);
}

static inline void kv_store(void* base, int type, size_t i, float v)
{
    if (type == LO_KV_F32) ((float*)base)[i] = v;
    else if (type == LO_KV_F16) ((uint16_t*)base)[i] = lo_f32_to_f16(v);
    else ((uint16_t*)base)[i] = lo_f32_to_bf16(v);
}

void lo_convert_from_f32(void* dst, int type, const float* src, size_t n)
{
    for (size_t i = 0; i < n; i++) kv_store(dst, type, i, src[i]);
}

void lo_convert_to_f32(float* dst, const void* src, int type, size_t n)
{
    for (size_t i = 0; i < n; i++) dst[i] = kv_load(src, type, i);
}

/* ---------------------------------------------------------------- math helpers ---------- */
/* rope_freq[i] = powf(base, -2i/rope_dim), fast/common.cpp:38-39 (rope_dim unclamped). */
void lo_rope_table(float* freq, int rope_dim, float base)
{
    for (int i = 0; i < rope_dim / 2; i++) freq[i] = powf(base, -2.0f * (float)i / (float)rope_dim);
}

/* fast/lil_math.cpp:901-920: adjacent pairs (i, i+1), rope_dim clamped to head_dim, made even. */
void lo_rope(float* x, int n_heads, int head_dim, int rope_dim, int pos, const float* freq)
{
    if (rope_dim > head_dim) rope_dim = head_dim;
    if (rope_dim & 1) rope_dim--;
    for (int h = 0; h < n_heads; h++) {
        float* v = x + (size_t)h * head_dim;
        for (int i = 0; i < rope_dim; i += 2) {
            const float ang = (float)pos * freq[i >> 1];
            const float c = cosf(ang), s = sinf(ang);
            const float x0 = v[i], x1 = v[i + 1];
            v[i] = x0 * c - x1 * s;
            v[i + 1] = x0 * s + x1 * c;
        }
    }
}

/* fast/lil_math.cpp:931-937 */
void lo_rmsnorm_inplace(float* x, const float* w, int n, float eps)
{
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    ss = 1.0f / sqrtf(ss / (float)n + eps);
    for (int i = 0; i < n; i++) x[i] = x[i] * ss * w[i];
}

/* fast/lil_math.cpp:964-976 */
void lo_softmax(float* x, int n)
{
    float mx = x[0];
    for (int i = 1; i < n; i++) if (x[i] > mx) mx = x[i];
    float sum = 0.0f;
    for (int i = 0; i < n; i++) { x[i] = expf(x[i] - mx); sum += x[i]; }
    for (int i = 0; i < n; i++) x[i] /= sum;
}

static inline float dot_f32(const float* a, const float* b, int n)
{
    float s = 0.0f;
    for (int i = 0; i < n; i++) s += a[i] * b[i];
    return s;
}

/* ---------------------------------------------------------------- decode ---------------- */
typedef struct lo_cfg {
    int n_heads;    /* q heads handled by this call (a SARA shard's q_headn) */
    int n_kv_heads; /* kv heads handled by this call (a shard's kv_headn) */
    int head_dim;
    int n_context;
    int rope_dim;   /* as gguf_model::rope_dim: clamped inside lo_rope */
    float eps;
    int qk_norm;
    int kv_type;
    int scale_mode; /* 0: score * (1/sqrtf(D)) (FAST), 1: score / sqrtf(D) (cpp, SARA) */
} lo_cfg;

/*
 * One layer of fast/ligguf_fast_qk.cpp:42-105.  kc/vc point at this layer's cache block
 * [n_context][kv_dim] (kv_dim = n_kv_heads*head_dim) of cfg->kv_type; q_in [H*D], k_in/v_in
 * [Hk*D] are the raw projections.  Writes the cache row `pos` and out [H*D].
 * Returns 0, or -1 on bad arguments.
 */
int lo_decode_layer(const lo_cfg* c, void* kc, void* vc, const float* freq, const float* qg,
                    const float* kg, int pos, const float* q_in, const float* k_in,
                    const float* v_in, float* out)
{
    const int H = c->n_heads, Hk = c->n_kv_heads, D = c->head_dim;
    if (H <= 0 || Hk <= 0 || H % Hk || D <= 0 || pos < 0 || pos >= c->n_context) return -1;
    const int kv_dim = Hk * D, nrep = H / Hk;
    float* q = (float*)malloc(sizeof(float) * (size_t)H * D);
    float* k = (float*)malloc(sizeof(float) * (size_t)kv_dim);
    float* v = (float*)malloc(sizeof(float) * (size_t)kv_dim);
    float* att = (float*)malloc(sizeof(float) * (size_t)H * (pos + 1));
    if (!q || !k || !v || !att) { free(q); free(k); free(v); free(att); return -1; }
    memcpy(q, q_in, sizeof(float) * (size_t)H * D);
    memcpy(k, k_in, sizeof(float) * (size_t)kv_dim);
    memcpy(v, v_in, sizeof(float) * (size_t)kv_dim);

    if (c->qk_norm) { /* fast/ligguf_fast_qk.cpp:42-51 */
        for (int h = 0; h < H; h++) lo_rmsnorm_inplace(q + (size_t)h * D, qg, D, c->eps);
        for (int h = 0; h < Hk; h++) lo_rmsnorm_inplace(k + (size_t)h * D, kg, D, c->eps);
    }
    lo_rope(q, H, D, c->rope_dim, pos, freq); /* :54-55 */
    lo_rope(k, Hk, D, c->rope_dim, pos, freq);

    const size_t row = (size_t)pos * kv_dim; /* :57-62 */
    for (int i = 0; i < kv_dim; i++) {
        kv_store(kc, c->kv_type, row + i, k[i]);
        kv_store(vc, c->kv_type, row + i, v[i]);
    }

    const float att_scale = 1.0f / sqrtf((float)D);
    const float att_div = sqrtf((float)D);
#pragma omp parallel for schedule(static)
    for (int h = 0; h < H; h++) { /* :66-105 */
        float* a = att + (size_t)h * (pos + 1);
        const float* qh = q + (size_t)h * D;
        const int g = h / nrep;
        for (int t = 0; t <= pos; t++) {
            float score;
            if (t == pos) score = dot_f32(qh, k + (size_t)g * D, D);
            else {
                const size_t base = (size_t)t * kv_dim + (size_t)g * D;
                score = 0.0f;
                for (int i = 0; i < D; i++) score += kv_load(kc, c->kv_type, base + i) * qh[i];
            }
            a[t] = c->scale_mode ? score / att_div : score * att_scale;
        }
        lo_softmax(a, pos + 1);
        float* xb = out + (size_t)h * D;
        for (int i = 0; i < D; i++) xb[i] = 0.0f;
        for (int t = 0; t <= pos; t++) {
            const float w = a[t];
            if (t == pos) {
                for (int i = 0; i < D; i++) xb[i] += w * v[(size_t)g * D + i];
            } else {
                const size_t base = (size_t)t * kv_dim + (size_t)g * D;
                for (int i = 0; i < D; i++) xb[i] += w * kv_load(vc, c->kv_type, base + i);
            }
        }
    }
    free(q); free(k); free(v); free(att);
    return 0;
}

/* Prefill as the reference performs it: one decode step per token (feed_text,
 * fast/ligguf_fast_qk.cpp:340-356).  q [n][H*D], k,v [n][Hk*D], out [n][H*D]. */
int lo_prefill_layer(const lo_cfg* c, void* kc, void* vc, const float* freq, const float* qg,
                     const float* kg, int pos0, int n, const float* q, const float* k,
                     const float* v, float* out)
{
    const size_t qd = (size_t)c->n_heads * c->head_dim, kd = (size_t)c->n_kv_heads * c->head_dim;
    for (int i = 0; i < n; i++) {
        const int rc = lo_decode_layer(c, kc, vc, freq, qg, kg, pos0 + i, q + i * qd, k + i * kd,
                                       v + i * kd, out + i * qd);
        if (rc) return rc;
    }
    return 0;
}

/*
 * fast/vdb.cpp:189-212 for a batch of padded sequences: sequence b has lens[b] tokens at rows
 * [b*max_len, b*max_len+lens[b]) of q/k/v/out, each row n_heads*head_dim wide.  Rows at or
 * beyond lens[b] are written as zeros.  Scale: multiply by 1/sqrtf(head_dim) (vdb.cpp:133,203).
 */
int lo_bert_attn(int n_heads, int head_dim, int batch, int max_len, const int* lens,
                 const float* q, const float* k, const float* v, float* out)
{
    const int E = n_heads * head_dim;
    const float att_scale = 1.0f / sqrtf((float)head_dim);
    for (int b = 0; b < batch; b++)
        if (lens[b] < 0 || lens[b] > max_len) return -1;
#pragma omp parallel for schedule(dynamic)
    for (int64_t bt = 0; bt < (int64_t)batch * max_len; bt++) {
        const int b = (int)(bt / max_len), t = (int)(bt % max_len);
        const int ntok = lens[b];
        float* ctx = out + (size_t)bt * E;
        for (int i = 0; i < E; i++) ctx[i] = 0.0f;
        if (t >= ntok) continue;
        float* att = (float*)malloc(sizeof(float) * (size_t)(ntok > 0 ? ntok : 1));
        const float* qrow = q + (size_t)bt * E;
        for (int h = 0; h < n_heads; h++) {
            float* ch = ctx + h * head_dim;
            const float* qh = qrow + h * head_dim;
            for (int tt = 0; tt < ntok; tt++) {
                const float* kh = k + ((size_t)b * max_len + tt) * E + h * head_dim;
                att[tt] = dot_f32(qh, kh, head_dim) * att_scale;
            }
            lo_softmax(att, ntok);
            for (int tt = 0; tt < ntok; tt++) {
                const float* vh = v + ((size_t)b * max_len + tt) * E + h * head_dim;
                const float a = att[tt];
                for (int i = 0; i < head_dim; i++) ch[i] += a * vh[i];
            }
        }
        free(att);
    }
    return 0;
}

/* ---------------------------------------------------------------- SARA shard map -------- */
/* cpp/ligguf_distrib.cpp:657-663 */
void lo_split_even(int total, int idx, int parts, int* off, int* count)
{
    const int base = total / parts, rem = total % parts;
    *count = base + (idx < rem);
    *off = idx * base + (idx < rem ? idx : rem);
}

/* ---------------------------------------------------------------- synthetic cache ------- */
/* Fills rows [pos0, pos0+n) of one layer's cache block (kv_dim_shard wide, kv_type) with the
 * generator's tensor `tensor` (LIGGUF_SYNTH_K=1 / _V=2), indexed by the unsharded element
 * row*kv_dim_full + kv_off + c, stream (tensor << 32) | layer - the indexing that
 * ligguf_cuda_attn_kv_synth uses. */
void lo_kv_synth(void* cache, int kv_type, int kv_dim_shard, int kv_dim_full, int kv_off,
                 int layer, int tensor, int pos0, int n, uint64_t seed, float scale)
{
    const uint64_t base = lo_synth_base(seed, ((uint64_t)tensor << 32) | (uint32_t)layer);
    const float mul = lo_synth_mul(scale);
#pragma omp parallel for schedule(static)
    for (int r = 0; r < n; r++) {
        const int t = pos0 + r;
        for (int c = 0; c < kv_dim_shard; c++) {
            const uint64_t idx = (uint64_t)t * (uint64_t)kv_dim_full + (uint64_t)(kv_off + c);
            kv_store(cache, kv_type, (size_t)t * kv_dim_shard + c, lo_synth_one(base, idx, mul, 0.0f));
        }
    }
}

/* OpenMP thread count of this library's parallel loops (a process launcher may have exported
 * OMP_NUM_THREADS=1 before the library loaded); returns the count now in effect. */
int lo_set_threads(int n)
{
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
#else
    (void)n;
    return 1;
#endif
}
