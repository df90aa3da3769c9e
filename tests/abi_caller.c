/* abi_caller.c - a plain C99 caller of include/ligguf_cuda_attn.h, linked against
 * libligguf_cuda_attn.so the way an engine binds it (test infrastructure).
 *
 *   abi_caller           argument checks that return before touching a GPU; prints "ok"
 *   abi_caller decode IN OUT
 *                        (GPU) one decode step of a Qwen3-shaped layer through the host-pointer
 *                        call, inputs from IN, the fp32 outputs to OUT
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "ligguf_cuda_attn.h"

#define CHECK(cond)                                                       \
    do {                                                                  \
        if (!(cond)) {                                                    \
            fprintf(stderr, "check failed: %s (line %d)\n", #cond, __LINE__); \
            return 1;                                                     \
        }                                                                 \
    } while (0)

static int no_gpu_checks(void)
{
    ligguf_attn* h = NULL;
    ligguf_attn_cfg c;
    memset(&c, 0, sizeof(c));
    CHECK(strcmp(ligguf_cuda_attn_strerror(LIGGUF_ATTN_EINVAL), "invalid argument") == 0);
    CHECK(ligguf_cuda_attn_init(NULL, &h) == LIGGUF_ATTN_EINVAL);
    c.n_layers = 1; c.n_heads = 6; c.n_kv_heads = 4; c.head_dim = 64; c.n_context = 16;
    CHECK(ligguf_cuda_attn_init(&c, &h) == LIGGUF_ATTN_EINVAL && h == NULL);
    CHECK(strlen(ligguf_cuda_attn_last_error()) > 0);
    CHECK(ligguf_cuda_attn_decode(NULL, 0, 0, NULL, NULL, NULL, NULL) == LIGGUF_ATTN_EINVAL);
    CHECK(ligguf_cuda_attn_state_save(NULL, "x", 1, NULL, 0) == LIGGUF_ATTN_EINVAL);
    CHECK(ligguf_cuda_attn_state_load(NULL, "x", NULL, NULL, NULL, 0) == LIGGUF_ATTN_EINVAL);
    CHECK(ligguf_cuda_bert_attn_tc_noalloc(12, 64, 1, LIGGUF_NOALLOC_MAX_ELEMS, (const int*)16, (const float*)16,
                                           (const float*)16, (const float*)16, (float*)16, NULL) == LIGGUF_ATTN_EINVAL);
    CHECK(ligguf_cuda_attn_free(NULL) == LIGGUF_ATTN_OK);
    return 0;
}

/* One decode step of a Qwen3-shaped layer (32 q / 8 KV heads, head_dim 128, QK norm, fp32 cache,
 * RoPE theta 1e6) at position POS through the host-pointer call, the engine's call site.  The
 * cache rows [0, POS) come from the library's seeded generator (seed 11, scale 1); the step's q,
 * k, v and the two norm weights are read from `in` (floats: q[H*D] k[HK*D] v[HK*D] qg[D] kg[D])
 * and the H*D outputs written to `out`. */
static int decode_case(const char* in, const char* out_path)
{
    enum { H = 32, HK = 8, D = 128, NCTX = 320, POS = 300 };
    static float buf[H * D + 2 * HK * D + 2 * D], out[H * D];
    const float *q = buf, *k = q + H * D, *v = k + HK * D, *qg = v + HK * D, *kg = qg + D;
    ligguf_attn_cfg c;
    ligguf_attn* h = NULL;
    FILE* f = fopen(in, "rb");
    CHECK(f && fread(buf, sizeof(buf), 1, f) == 1);
    fclose(f);
    memset(&c, 0, sizeof(c));
    c.n_layers = 1; c.n_heads = H; c.n_kv_heads = HK; c.head_dim = D; c.n_context = NCTX;
    c.rope_dim = D; c.rope_base = 1e6f; c.rms_epsilon = 1e-6f; c.qk_norm = 1;
    c.kv_type = LIGGUF_KV_F32; c.scale_mode = LIGGUF_SCALE_MUL;
    CHECK(ligguf_cuda_attn_init(&c, &h) == 0);
    CHECK(ligguf_cuda_attn_set_qk_norm(h, 0, qg, kg) == 0);
    CHECK(ligguf_cuda_attn_kv_synth(h, 0, 1, 0, POS, 11, 1.0f) == 0);
    CHECK(ligguf_cuda_attn_decode(h, 0, POS, q, k, v, out) == 0);
    CHECK(ligguf_cuda_attn_free(h) == 0);
    f = fopen(out_path, "wb");
    CHECK(f && fwrite(out, sizeof(out), 1, f) == 1);
    fclose(f);
    return 0;
}

int main(int argc, char** argv)
{
    if (argc > 3 && strcmp(argv[1], "decode") == 0) return decode_case(argv[2], argv[3]);
    if (no_gpu_checks()) return 1;
    puts("ok");
    return 0;
}
