/*
 * qmat_oracle.c - plain-C restatement of the reference's QKV projection arithmetic (the "port"):
 * the activation quantizers and the per-type row dots of matmul / matmul3.
 *
 * TEST INFRASTRUCTURE ONLY: the CPU checker of the CUDA kernels in ligguf_b200/csrc/qmatvec.cuh,
 * built into liboracle_port.so by oracle/Makefile, never linked into the product.
 *
 * Follows (matrixsmaster/ligguf):
 *   quantize_q8_K  fast/lil_math.cpp:352-385   quantize_q8_0  fast/lil_math.cpp:329-350
 *   matmul         fast/lil_math.cpp:757-778   matmul3        fast/lil_math.cpp:827-899
 *   dot_q8_0_q8_0 :408-419, dot_q8_0_q1_0 :421-438, dot_q8_0_q1_G :440-466, dot_q8_K_q2_K :548-578,
 *   dot_q8_K_q3_K :468-546, dot_q8_K_q4_K :580-616, dot_q8_K_q5_K :618-694, dot_q8_K_q6_K :696-742,
 *   dot_f32 / dot_f16_f32 :389-406 (the scalar forms of the AVX2 code in fast/arch_avx2.h:83-435),
 *   block layouts fast/lil_gguf.h:64-119, get_scale_min_k4 fast/lil_math.cpp:139-149.
 * The reference is built with -Ofast; measured against that build (tests/test_oracle_qmat.py), its
 * quantizers compute quantize_q8_0's d as amax * (1/127) and its 1/d as 127/amax, and quantize_q8_K's
 * d as max * (-1/127) (the compiler folds 1/(-127/max)), while -127/max stays an IEEE division.
 * This file uses those forms, built with -ffp-contract=off.  The row dots sum block terms in the
 * scalar order.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

float lo_f16_to_f32(uint16_t h);
uint16_t lo_f32_to_f16(float f);

enum { T_F32 = 0, T_F16 = 1, T_Q8_0 = 8, T_Q2_K = 10, T_Q3_K = 11, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14,
       T_Q1_0 = 40, T_Q1_G = 41 };

typedef struct { float d; int8_t qs[256]; int16_t bsums[16]; } q8k_t;      /* 292 bytes */
typedef struct { uint16_t d; int8_t qs[32]; } __attribute__((packed)) q80_t; /* 34 bytes */

static int nearest(float f) { return f < 0.f ? (int)(f - 0.5f) : (int)(f + 0.5f); }

void lo_quantize_q8_K(const float* x, int n, void* out)
{
    q8k_t* y = (q8k_t*)out;
    for (int b = 0; b < n / 256; b++) {
        const float* p = x + 256 * b;
        float amax = 0.f, mx = 0.f;
        for (int j = 0; j < 256; j++) {
            const float ax = fabsf(p[j]);
            if (ax > amax) { amax = ax; mx = p[j]; }
        }
        if (amax == 0.f) {
            memset(&y[b], 0, sizeof(q8k_t));
            continue;
        }
        const float iscale = -127.0f / mx;
        for (int j = 0; j < 256; j++) {
            const int v = nearest(iscale * p[j]);
            y[b].qs[j] = (int8_t)(v < 127 ? v : 127);
        }
        for (int g = 0; g < 16; g++) {
            int s = 0;
            for (int i = 0; i < 16; i++) s += y[b].qs[16 * g + i];
            y[b].bsums[g] = (int16_t)s;
        }
        y[b].d = mx * (-1.0f / 127.0f);
    }
}

void lo_quantize_q8_0(const float* x, int n, void* out)
{
    q80_t* y = (q80_t*)out;
    for (int b = 0; b < n / 32; b++) {
        float amax = 0.f;
        for (int j = 0; j < 32; j++) {
            const float a = fabsf(x[32 * b + j]);
            if (a > amax) amax = a;
        }
        const float d = amax * (1.0f / 127.0f);
        const float id = d != 0.f ? 127.0f / amax : 0.f;
        y[b].d = lo_f32_to_f16(d);
        for (int j = 0; j < 32; j++) y[b].qs[j] = (int8_t)roundf(x[32 * b + j] * id);
    }
}

static float h(const uint8_t* p) { uint16_t v; memcpy(&v, p, 2); return lo_f16_to_f32(v); }

static void k4_scale_min(int j, const uint8_t* q, int* sc, int* m)
{
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

/* One row: weights `w` (GGUF blocks of `type`) against x (fp32), its Q8_K form yk, its Q8_0 form y0. */
static float row_dot(int type, const uint8_t* w, const float* x, const q8k_t* yk, const q80_t* y0, int n)
{
    float acc = 0.f;
    switch (type) {
    case T_F32:
        for (int i = 0; i < n; i++) { float v; memcpy(&v, w + 4 * i, 4); acc += v * x[i]; }
        return acc;
    case T_F16:
        for (int i = 0; i < n; i++) acc += h(w + 2 * i) * x[i];
        return acc;
    case T_Q8_0:
        for (int b = 0; b < n / 32; b++) {
            const uint8_t* blk = w + 34 * b;
            int s = 0;
            for (int j = 0; j < 32; j++) s += (int8_t)blk[2 + j] * y0[b].qs[j];
            acc += h(blk) * lo_f16_to_f32(y0[b].d) * (float)s;
        }
        return acc;
    case T_Q1_0:
        for (int b = 0; b < n / 32; b++) {
            const uint8_t* blk = w + 6 * b;
            int s = 0;
            for (int j = 0; j < 32; j++) s += (((blk[2 + (j >> 3)] >> (j & 7)) & 1) ? 1 : -1) * y0[b].qs[j];
            acc += h(blk) * lo_f16_to_f32(y0[b].d) * (float)s;
        }
        return acc;
    case T_Q1_G:
        for (int b = 0; b < n / 128; b++) {
            const uint8_t* blk = w + 18 * b;
            float si = 0.f;
            for (int k = 0; k < 4; k++) {
                const q80_t* yb = &y0[4 * b + k];
                int s = 0;
                for (int j = 0; j < 32; j++) {
                    const int bit = 32 * k + j;
                    s += (((blk[2 + (bit >> 3)] >> (bit & 7)) & 1) ? 1 : -1) * yb->qs[j];
                }
                si += lo_f16_to_f32(yb->d) * (float)s;
            }
            acc += h(blk) * si;
        }
        return acc;
    case T_Q2_K:
        for (int b = 0; b < n / 256; b++) {
            const uint8_t* blk = w + 84 * b;
            const uint8_t* sc = blk;
            const int8_t* q8 = yk[b].qs;
            int summs = 0, isum = 0;
            for (int g = 0; g < 16; g++) summs += yk[b].bsums[g] * (sc[g] >> 4);
            for (int e = 0; e < 256; e++) {  /* element e: byte 32*(e/128) + e%32, shift 2*((e%128)/32) */
                const int q = (blk[16 + 32 * (e / 128) + e % 32] >> (2 * ((e % 128) / 32))) & 3;
                isum += (sc[e / 16] & 0xF) * q * q8[e];
            }
            acc += yk[b].d * h(blk + 80) * (float)isum - yk[b].d * h(blk + 82) * (float)summs;
        }
        return acc;
    case T_Q3_K:
        for (int b = 0; b < n / 256; b++) {
            const uint8_t* blk = w + 110 * b;
            const uint8_t* sb = blk + 96;
            int sc[16];
            for (int g = 0; g < 16; g++) {  /* the 12-byte packing of 16 six-bit scales */
                const int i = g & 3, lo = (g & 4) ? sb[4 + i] : sb[i];
                sc[g] = (((g & 8) ? (lo >> 4) : (lo & 0xF)) | (((sb[8 + i] >> (2 * (g >> 2))) & 3) << 4)) - 32;
            }
            int isum = 0;
            for (int e = 0; e < 256; e++) {
                const int k = e / 128, j = (e % 128) / 32, l = e % 32;
                int q = (blk[32 + 32 * k + l] >> (2 * j)) & 3;
                if (!(blk[l] & (1 << (4 * k + j)))) q -= 4;
                isum += sc[e / 16] * q * yk[b].qs[e];
            }
            acc += h(blk + 108) * yk[b].d * (float)isum;
        }
        return acc;
    case T_Q4_K:
        for (int b = 0; b < n / 256; b++) {
            const uint8_t* blk = w + 144 * b;
            const float d = h(blk) * yk[b].d, dmin = h(blk + 2) * yk[b].d;
            for (int s = 0; s < 8; s++) {
                int sc, m, dot = 0;
                k4_scale_min(s, blk + 4, &sc, &m);
                for (int l = 0; l < 32; l++) {
                    const uint8_t q = blk[16 + 32 * (s / 2) + l];
                    dot += yk[b].qs[32 * s + l] * ((s & 1) ? (q >> 4) : (q & 0xF));
                }
                acc += d * sc * dot - dmin * m * (yk[b].bsums[2 * s] + yk[b].bsums[2 * s + 1]);
            }
        }
        return acc;
    case T_Q5_K:
        for (int b = 0; b < n / 256; b++) {
            const uint8_t* blk = w + 176 * b;
            int sumi = 0, isum = 0;
            for (int s = 0; s < 8; s++) {
                int sc, m;
                k4_scale_min(s, blk + 4, &sc, &m);
                sumi += m * (yk[b].bsums[2 * s] + yk[b].bsums[2 * s + 1]);
                for (int l = 0; l < 32; l++) {
                    const uint8_t q = blk[48 + 32 * (s / 2) + l];
                    const int v = ((s & 1) ? (q >> 4) : (q & 0xF)) + (((blk[16 + l] >> s) & 1) ? 16 : 0);
                    isum += sc * v * yk[b].qs[32 * s + l];
                }
            }
            acc += h(blk) * yk[b].d * (float)isum - h(blk + 2) * yk[b].d * (float)sumi;
        }
        return acc;
    case T_Q6_K:
        for (int b = 0; b < n / 256; b++) {
            const uint8_t* blk = w + 210 * b;
            const int8_t* sc = (const int8_t*)(blk + 192);
            int isum = 0;
            for (int e = 0; e < 256; e++) {
                const int c = e / 128, qq = (e % 128) / 32, l = e % 32;
                const uint8_t lo = blk[64 * c + 32 * (qq & 1) + l];
                const uint8_t hi = blk[128 + 32 * c + l];
                const int v = (((qq >> 1) ? (lo >> 4) : (lo & 0xF)) | (((hi >> (2 * qq)) & 3) << 4)) - 32;
                isum += sc[e / 16] * v * yk[b].qs[e];
            }
            acc += h(blk + 208) * yk[b].d * (float)isum;
        }
        return acc;
    default:
        return NAN;
    }
}

/* out[r] = row r of w (d rows of rb bytes) against x, with x quantized as matmul3 does. */
void lo_matmul(float* out, const float* x, int n, int type, const void* w, int rb, int d, void* scratch_k,
               void* scratch_0)
{
    q8k_t* yk = (q8k_t*)scratch_k;
    q80_t* y0 = (q80_t*)scratch_0;
    if (n % 256 == 0) lo_quantize_q8_K(x, n, yk);
    if (n % 32 == 0) lo_quantize_q8_0(x, n, y0);
#pragma omp parallel for schedule(static)
    for (int r = 0; r < d; r++) out[r] = row_dot(type, (const uint8_t*)w + (size_t)r * rb, x, yk, y0, n);
}
