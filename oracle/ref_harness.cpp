/*
 * ref_harness.cpp - runs the REFERENCE's own math (fast/lil_math.cpp of matrixsmaster/ligguf,
 * compiled from its source by oracle/Makefile with the reference's flags) through the loop of
 * its attention block, so that the C restatement in attn_oracle.c and the golden fixtures can be
 * checked against the reference's arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY (built into oracle/_ref/, never linked into the product).
 *
 * The engine itself cannot run here: inference() needs a GGUF model file and none is available,
 * so this harness restates the loop around the reference's functions:
 *   rf_decode_layer   fast/ligguf_fast_qk.cpp:42-105, calling rmsnorm_inplace (lil_math.cpp:931),
 *                     rope (lil_math.cpp:901), f32_to_f16_row (lil_math.cpp:83), vec_dot_f32 /
 *                     vec_dot_f16_f32 (lil_math.cpp:319-327 -> AVX2 dot_f32/dot_f16_f32,
 *                     arch_avx2.h:83-109), softmax (lil_math.cpp:964) and the fp16 LUT
 *                     (lil_math.h:5).  With an fp32 cache (the cpp/ligguf.cpp:674-718 layout) the
 *                     cached rows go through vec_dot_f32 instead of vec_dot_f16_f32.
 *   rf_bert_attn      fast/vdb.cpp:189-212 with vec_dot_f32 and softmax.
 * The FAST block runs heads under `omp parallel for` (MULTITHREAD, fast/common.h:11); so does
 * this harness.  bert_embed has no threading; neither does rf_bert_attn.
 */
#include <math.h>
#include <string.h>
#include <vector>

#include <omp.h>

#include "lil_gguf.h"
#include "lil_math.h"

struct rf_cfg { /* same layout as lo_cfg in attn_oracle.c */
    int n_heads;
    int n_kv_heads;
    int head_dim;
    int n_context;
    int rope_dim;
    float eps;
    int qk_norm;
    int kv_type; /* 0 = fp32 cache, 1 = fp16 cache (the reference has no bf16 cache) */
    int scale_mode;
};

static bool g_lut_ready = false;

extern "C" void rf_init(void)
{
    if (!g_lut_ready) {
        fp1632_init();
        g_lut_ready = true;
    }
}

/* The reference's fp32 -> fp16 row conversion (f32_to_f16_row, lil_math.cpp:83-86). */
extern "C" void rf_f32_to_f16_row(const float* x, uint16_t* y, int n) { f32_to_f16_row(x, y, n); }
extern "C" float rf_fp16_to_fp32(uint16_t h)
{
    rf_init();
    return fp16_to_fp32(h);
}
extern "C" void rf_softmax(float* x, int n) { softmax(x, n); }
extern "C" void rf_rmsnorm_inplace(float* x, const float* w, int n, float eps)
{
    rmsnorm_inplace(x, const_cast<float*>(w), n, eps);
}
extern "C" void rf_rope(float* x, int n_heads, int head_dim, int rope_dim, int pos,
                        const float* freq)
{
    gguf_model m;
    m.head_dim = head_dim;
    m.rope_dim = rope_dim;
    ftensor v(x, x + (size_t)n_heads * head_dim);
    ftensor f(freq, freq + (rope_dim > 0 ? rope_dim / 2 : 0));
    rope(v, n_heads, pos, m, f);
    memcpy(x, v.data(), sizeof(float) * v.size());
}

extern "C" int rf_decode_layer(const rf_cfg* c, void* kc_layer, void* vc_layer, const float* freq,
                               const float* qg, const float* kg, int pos, const float* q_in,
                               const float* k_in, const float* v_in, float* out)
{
    rf_init();
    const int H = c->n_heads, Hk = c->n_kv_heads, D = c->head_dim;
    if (H <= 0 || Hk <= 0 || H % Hk || pos < 0 || pos >= c->n_context) return -1;
    if (c->kv_type != 0 && c->kv_type != 1) return -1;
    const int kv_dim = Hk * D;
    const float att_scale = 1.0f / sqrtf(D);

    gguf_model m;
    m.head_dim = D;
    m.rope_dim = c->rope_dim;
    ftensor rope_freq(freq, freq + (c->rope_dim > 0 ? c->rope_dim / 2 : 0));
    ftensor q(q_in, q_in + (size_t)H * D), k(k_in, k_in + kv_dim), v(v_in, v_in + kv_dim);
    std::vector<float> att((size_t)H * (pos + 1));

    if (c->qk_norm) {
        float* p = q.data();
        for (int h = 0; h < H; h++, p += D) rmsnorm_inplace(p, const_cast<float*>(qg), D, c->eps);
        p = k.data();
        for (int h = 0; h < Hk; h++, p += D) rmsnorm_inplace(p, const_cast<float*>(kg), D, c->eps);
    }
    rope(q, H, pos, m, rope_freq);
    rope(k, Hk, pos, m, rope_freq);

    if (c->kv_type == 1) {
        gguf_half* kc = (gguf_half*)kc_layer;
        gguf_half* vc = (gguf_half*)vc_layer;
        f32_to_f16_row(k.data(), kc + (size_t)pos * kv_dim, kv_dim);
        f32_to_f16_row(v.data(), vc + (size_t)pos * kv_dim, kv_dim);
    } else {
        memcpy((float*)kc_layer + (size_t)pos * kv_dim, k.data(), sizeof(float) * kv_dim);
        memcpy((float*)vc_layer + (size_t)pos * kv_dim, v.data(), sizeof(float) * kv_dim);
    }

    const int nrep = H / Hk;
#pragma omp parallel for
    for (int h = 0; h < H; h++) {
        float* a = att.data() + (size_t)h * (pos + 1);
        float* qh = q.data() + (size_t)h * D;
        float* kh = k.data() + (size_t)(h / nrep) * D;
        float* vh = v.data() + (size_t)(h / nrep) * D;
        for (int t = 0; t <= pos; t++) {
            float score;
            if (t == pos) score = vec_dot_f32(qh, kh, D);
            else if (c->kv_type == 1)
                score = vec_dot_f16_f32((gguf_half*)kc_layer + (size_t)t * kv_dim + (h / nrep) * D, qh, D);
            else
                score = vec_dot_f32((float*)kc_layer + (size_t)t * kv_dim + (h / nrep) * D, qh, D);
            a[t] = c->scale_mode ? score / sqrtf(D) : score * att_scale;
        }
        softmax(a, pos + 1);
        float* xb = out + (size_t)h * D;
        memset(xb, 0, sizeof(float) * D);
        for (int t = 0; t <= pos; t++) {
            const float w = a[t];
            if (t == pos) {
                for (int i = 0; i < D; i++) xb[i] += w * vh[i];
            } else if (c->kv_type == 1) {
                const gguf_half* vr = (gguf_half*)vc_layer + (size_t)t * kv_dim + (h / nrep) * D;
                for (int i = 0; i < D; i++) xb[i] += w * fp16_to_fp32(vr[i]);
            } else {
                const float* vr = (float*)vc_layer + (size_t)t * kv_dim + (h / nrep) * D;
                for (int i = 0; i < D; i++) xb[i] += w * vr[i];
            }
        }
    }
    return 0;
}

extern "C" int rf_prefill_layer(const rf_cfg* c, void* kc, void* vc, const float* freq,
                                const float* qg, const float* kg, int pos0, int n, const float* q,
                                const float* k, const float* v, float* out)
{
    const size_t qd = (size_t)c->n_heads * c->head_dim, kd = (size_t)c->n_kv_heads * c->head_dim;
    for (int i = 0; i < n; i++) {
        const int rc = rf_decode_layer(c, kc, vc, freq, qg, kg, pos0 + i, q + i * qd, k + i * kd,
                                       v + i * kd, out + i * qd);
        if (rc) return rc;
    }
    return 0;
}

extern "C" int rf_bert_attn(int n_heads, int head_dim, int batch, int max_len, const int* lens,
                            const float* q, const float* k, const float* v, float* out)
{
    const int n_embed = n_heads * head_dim;
    const float att_scale = 1.0f / sqrtf(head_dim);
    std::vector<float> att(max_len > 0 ? max_len : 1);
    for (int b = 0; b < batch; b++) {
        const int ntok = lens[b];
        if (ntok < 0 || ntok > max_len) return -1;
        const size_t b0 = (size_t)b * max_len * n_embed;
        for (int t = 0; t < max_len; t++) {
            float* ctx = out + b0 + (size_t)t * n_embed;
            for (int i = 0; i < n_embed; i++) ctx[i] = 0.0f;
            if (t >= ntok) continue;
            const float* qt = q + b0 + (size_t)t * n_embed;
            for (int h = 0; h < n_heads; h++) {
                float* ch = ctx + h * head_dim;
                const float* qh = qt + h * head_dim;
                for (int tt = 0; tt < ntok; tt++) {
                    const float* kh = k + b0 + (size_t)tt * n_embed + h * head_dim;
                    att[tt] = vec_dot_f32(qh, kh, head_dim) * att_scale;
                }
                softmax(att.data(), ntok);
                for (int tt = 0; tt < ntok; tt++) {
                    const float* vh = v + b0 + (size_t)tt * n_embed + h * head_dim;
                    const float a = att[tt];
                    for (int i = 0; i < head_dim; i++) ch[i] += a * vh[i];
                }
            }
        }
    }
    return 0;
}

/* Thread count of the `omp parallel for` over heads (the reference's MULTITHREAD), whatever
 * OMP_NUM_THREADS the process was started with; returns the count now in effect. */
extern "C" int rf_set_threads(int n)
{
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
}

/* ---- the QKV projection (matmul3, lil_math.cpp:827-899) and its activation quantizers ------- */
/* quantize_q8_K (lil_math.cpp:352-385): n/256 blocks {float d; int8 qs[256]; int16 bsums[16]},
 * 292 bytes each, written to `out` in the struct's layout. */
extern "C" void rf_quantize_q8_K(const float* x, int n, void* out)
{
    ftensor xv(x, x + n);
    ktensor y(n / QK_K);
    quantize_q8_K(y, xv);
    memcpy(out, y.data(), y.size() * sizeof(block_q8_K));
}
/* quantize_q8_0 (lil_math.cpp:329-350): n/32 blocks {fp16 d; int8 qs[32]}, 34 bytes each. */
extern "C" void rf_quantize_q8_0(const float* x, int n, void* out)
{
    ftensor xv(x, x + n);
    qtensor y(n / QK8_0);
    quantize_q8_0(y, xv);
    memcpy(out, y.data(), y.size() * sizeof(block_q8_0));
}
/* The engine's QKV step (fast/ligguf_fast_qk.cpp:39-40): quantize_q8_K of the normed activation,
 * then matmul3 over three weight matrices of GGUF type t0..t2 (rows of rsz0..2 bytes). */
extern "C" void rf_matmul3(float* out0, float* out1, float* out2, const float* x, int n, int t0, const void* w0,
                           int rsz0, int d0, int t1, const void* w1, int rsz1, int d1, int t2, const void* w2,
                           int rsz2, int d2)
{
    rf_init();
    ftensor xv(x, x + n), o0(d0), o1(d1), o2(d2);
    ktensor xq(n / QK_K > 0 ? n / QK_K : 1);
    if (n % QK_K == 0) quantize_q8_K(xq, xv);
    wtensor a = {(uint8_t*)w0, (gguf_type)t0, (uint32_t)rsz0};
    wtensor b = {(uint8_t*)w1, (gguf_type)t1, (uint32_t)rsz1};
    wtensor c = {(uint8_t*)w2, (gguf_type)t2, (uint32_t)rsz2};
    matmul3(o0, o1, o2, &xv, &xq, NULL, a, b, c, n, d0, d1, d2);
    memcpy(out0, o0.data(), d0 * sizeof(float));
    memcpy(out1, o1.data(), d1 * sizeof(float));
    memcpy(out2, o2.data(), d2 * sizeof(float));
}
/* matmul (lil_math.cpp) over one matrix: the attn_output projection of the block
 * (fast/ligguf_fast_qk.cpp:108-109). */
extern "C" void rf_matmul(float* out, const float* x, int n, int t, const void* w, int rsz, int d)
{
    rf_init();
    ftensor xv(x, x + n), o(d);
    ktensor xq(n / QK_K > 0 ? n / QK_K : 1);
    if (n % QK_K == 0) quantize_q8_K(xq, xv);
    wtensor a = {(uint8_t*)w, (gguf_type)t, (uint32_t)rsz};
    matmul(o, &xv, &xq, NULL, a, n, d);
    memcpy(out, o.data(), d * sizeof(float));
}
