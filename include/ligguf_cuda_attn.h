/*
 * ligguf_cuda_attn.h - C ABI of the B200 (sm_100a) attention block for LiGGUF's FAST engine.
 *
 * The reference engine has no plugin or FFI layer for attention: the block is inline code in
 * `void inference(int tok)` (fast/ligguf_fast_qk.cpp:24-105) working on the global
 * `model_state g_m` (fast/common.h:33-74).  This header is the drop-in boundary that replaces
 * that inline block: plain C types, plain pointers and sizes, int status codes, no torch and
 * no CUDA types in any signature (streams and IPC handles travel as `void*`).
 *
 * Conventions (mirroring the reference's):
 *   - one host thread drives one handle, like `inference()` is driven by one thread
 *     (fast/ligguf_fast_qk.cpp:316-322); a handle is not re-entrant and its kernels of one
 *     call must not overlap on the GPU with those of another call on the same handle;
 *   - `pos` is explicit on every call (the reference keeps it in g_m.pos and increments it at
 *     fast/ligguf_fast_qk.cpp:27); rewinding (kv_backtrack, fast/ligguf_fast_qk.cpp:333-338)
 *     is therefore just passing a smaller pos;
 *   - errors never abort: every entry point returns 0 or a negative LIGGUF_ATTN_E* code, and
 *     ligguf_cuda_attn_last_error() gives a one-line reason (the reference prints with ERR,
 *     fast/common.h:14, or asserts).
 */
#ifndef LIGGUF_CUDA_ATTN_H
#define LIGGUF_CUDA_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------------------------- */
#define LIGGUF_ATTN_OK 0
#define LIGGUF_ATTN_EINVAL (-1)      /* bad argument (NULL, out-of-range layer/pos, bad dims) */
#define LIGGUF_ATTN_ECUDA (-2)       /* a CUDA runtime call failed */
#define LIGGUF_ATTN_ENOMEM (-3)      /* device or pinned host allocation failed */
#define LIGGUF_ATTN_ETIMEDOUT (-4)   /* a bounded in-kernel wait gave up (kernel returned early) */
#define LIGGUF_ATTN_EUNSUPPORTED (-5)/* shape/type combination without a kernel */
#define LIGGUF_ATTN_ESTATE (-6)      /* call not valid in the handle's current state */

/* ---- enums ----------------------------------------------------------------------------- */
/* KV-cache element type.  FAST stores fp16 (`htensor kc, vc`, fast/common.h:60, written with
 * f32_to_f16_row at fast/ligguf_fast_qk.cpp:61-62); the single-file engines store fp32
 * (cpp/ligguf.cpp:674-679, cpp/ligguf_distrib.cpp:724-727).  bf16 has no reference
 * counterpart and exists for the tensor-core prefill path. */
#define LIGGUF_KV_F32 0
#define LIGGUF_KV_F16 1
#define LIGGUF_KV_BF16 2

/* Score scaling.  FAST multiplies by att_scale = 1/sqrtf(head_dim)
 * (fast/ligguf_fast_qk.cpp:26,85; fast/vdb.cpp:133,203); the cpp/c/SARA engines divide by
 * sqrtf(head_dim) (cpp/ligguf.cpp:696, c/ligguf.c, cpp/ligguf_distrib.cpp:735). */
#define LIGGUF_SCALE_MUL 0
#define LIGGUF_SCALE_DIV 1

/* Prefill / BERT arithmetic: fp32 on CUDA cores (tight-tolerance path) or bf16 operands on
 * the tcgen05 tensor cores with fp32 accumulation. */
#define LIGGUF_MODE_SIMT 0
#define LIGGUF_MODE_TC 1

/* ---- decoder attention handle ---------------------------------------------------------- */
typedef struct ligguf_attn_cfg {
    int n_layers;        /* gguf_model::n_layers (fast/lil_gguf.h:166) */
    int n_heads;         /* query heads of the whole model (gguf_model::n_heads) */
    int n_kv_heads;      /* KV heads of the whole model (gguf_model::n_kv_heads) */
    int head_dim;        /* gguf_model::head_dim; 64 or 128 */
    int n_context;       /* cache positions per layer (gguf_model::n_context after allocate(),
                            fast/common.cpp:13-19) */
    int rope_dim;        /* gguf_model::rope_dim; clamped to head_dim and made even exactly as
                            rope() does (fast/lil_math.cpp:904-906); 0 = no RoPE */
    float rope_base;     /* gguf_model::rope_base (theta) */
    const float* rope_freq; /* optional host table of rope_dim/2 inverse frequencies
                            (model_state::rope_freq, fast/common.cpp:34,38-39); NULL = the
                            library computes powf(rope_base, -2i/rope_dim) the same way */
    float rms_epsilon;   /* gguf_model::rms_epsilon, used by the Qwen3 QK norm */
    int qk_norm;         /* 1 = per-head RMSNorm of q and k before RoPE (arch "qwen3",
                            fast/ligguf_fast_qk.cpp:42-51) */
    int kv_type;         /* LIGGUF_KV_* */
    int scale_mode;      /* LIGGUF_SCALE_* */
    int device;          /* CUDA device ordinal the cache lives on */
    int kv_head0;        /* SARA shard: first KV head owned (shard_desc::kv_head0,
                            cpp/ligguf_distrib.cpp:120-124,665-679); 0 when unsharded */
    int kv_headn;        /* SARA shard: KV heads owned; 0 = all n_kv_heads */
} ligguf_attn_cfg;

typedef struct ligguf_attn ligguf_attn;

/* Replaces the attention part of model_state::allocate() (fast/common.cpp:31-39): allocates the
 * HBM-resident cache [n_layers][n_context][kv_headn*head_dim] (zero-filled, the reference's
 * kc.resize(...,0)), the RoPE table and per-layer QK-norm weights.  The q heads owned are
 * [kv_head0*nrep, (kv_head0+kv_headn)*nrep), nrep = n_heads/n_kv_heads
 * (cpp/ligguf_distrib.cpp:668-669). */
int ligguf_cuda_attn_init(const ligguf_attn_cfg* cfg, ligguf_attn** out);
int ligguf_cuda_attn_free(ligguf_attn* h);
const char* ligguf_cuda_attn_strerror(int status);
/* One-line reason for the last failure on the calling host thread ("" if none). */
const char* ligguf_cuda_attn_last_error(void);

/* Device-resident copies of one layer's attn_q_norm / attn_k_norm weights (head_dim floats each,
 * host pointers; gguf trans_block::att_q_norm/att_k_norm, fast/lil_gguf.h:138-139).  Required
 * for every layer when cfg.qk_norm is set. */
int ligguf_cuda_attn_set_qk_norm(ligguf_attn* h, int layer, const float* q_gamma,
                                 const float* k_gamma);

/* One decode step of one layer: replaces fast/ligguf_fast_qk.cpp:42-105.
 *   q   [q_headn*head_dim]  raw projection output g_m.q (pre norm, pre RoPE)
 *   k,v [kv_headn*head_dim] raw g_m.k / g_m.v
 *   out [q_headn*head_dim]  attention result, the reference's g_m.xb
 * Applies QK norm (if enabled) and RoPE at `pos`, appends k,v to the cache row `pos`, and
 * attends over positions [0, pos] with position `pos` taken from the fp32 k,v as FAST does
 * (fast/ligguf_fast_qk.cpp:77-78,98-99).  Host pointers; returns when `out` is written. */
int ligguf_cuda_attn_decode(ligguf_attn* h, int layer, int pos, const float* q, const float* k,
                            const float* v, float* out);
/* Same with device pointers, enqueued on `stream` (a cudaStream_t; NULL = legacy default). */
int ligguf_cuda_attn_decode_async(ligguf_attn* h, int layer, int pos, const float* d_q,
                                  const float* d_k, const float* d_v, float* d_out,
                                  void* stream);

/* Causal prefill of n tokens at positions [pos0, pos0+n) of one layer.  The reference has no
 * batched prefill: feed_text() runs inference() once per token (fast/ligguf_fast_qk.cpp:340-356),
 * so the result equals n decode calls at pos0..pos0+n-1.
 *   q [n][q_headn*head_dim], k,v [n][kv_headn*head_dim] raw; out [n][q_headn*head_dim].
 * mode: LIGGUF_MODE_SIMT (fp32) or LIGGUF_MODE_TC (bf16 tcgen05, fp32 accumulate). */
int ligguf_cuda_attn_prefill(ligguf_attn* h, int layer, int pos0, int n, const float* q,
                             const float* k, const float* v, float* out, int mode);
/* Same with device pointers on `stream`; d_q, d_k and d_v must be 16-byte aligned (their rows are
 * bulk-copied), else LIGGUF_ATTN_EINVAL. */
int ligguf_cuda_attn_prefill_async(ligguf_attn* h, int layer, int pos0, int n, const float* d_q,
                                   const float* d_k, const float* d_v, float* d_out, int mode,
                                   void* stream);

/* Cache rows [pos0, pos0+n) of one layer, in the handle's kv_type, row layout
 * [n][kv_headn*head_dim] - with kv_type F16 this is byte-for-byte the per-layer block that
 * save_model_state/load_model_state write and read (fast/ligguf_fast_qk.cpp:236-247,288-295). */
int ligguf_cuda_attn_kv_download(ligguf_attn* h, int layer, int pos0, int n, void* host_k,
                                 void* host_v);
int ligguf_cuda_attn_kv_upload(ligguf_attn* h, int layer, int pos0, int n, const void* host_k,
                               const void* host_v);
/* FAST engine state file (`model_file`, fast/common.h:26-31) straight from / into the HBM cache,
 * byte for byte what save_model_state / load_model_state write and read
 * (fast/ligguf_fast_qk.cpp:216-302): the packed 24-byte header {int pos; int n_context;
 * uint64_t kv_size; uint64_t logits_size}, then for K and then V, each layer's rows [0, pos) as
 * [pos][kv_dim] fp16, then logits_size fp32 logits.  The handle must hold the whole model (no SARA
 * shard) with kv_type LIGGUF_KV_F16, the format's element type.
 *   save: `pos` cached rows (1 <= pos <= n_context) and the caller's `logits` (host, n_logits
 *         floats; the reference saves nothing when pos or the logits are empty).
 *   load: checks the header as the reference does (non-zero sizes, kv_size = n_layers*pos*kv_dim,
 *         logits_size = n_logits) and that pos fits the handle's n_context; uploads the rows and
 *         fills `logits`; *pos_out / *n_context_out (either may be NULL) get the header's values.
 *         A file that fails a check leaves the cache and `logits` untouched (LIGGUF_ATTN_EINVAL).
 * Synchronous; errors in opening, reading or writing the file return LIGGUF_ATTN_EINVAL. */
int ligguf_cuda_attn_state_save(ligguf_attn* h, const char* path, int pos, const float* logits,
                                uint64_t n_logits);
int ligguf_cuda_attn_state_load(ligguf_attn* h, const char* path, int* pos_out, int* n_context_out,
                                float* logits, uint64_t n_logits);
/* Fills cache rows [pos0, pos0+n) of layers [layer0, layer0+n_layers) with the library's seeded
 * synthetic generator (ligguf_cuda_synth_fill, tensor ids LIGGUF_SYNTH_K / _V), indexed by the
 * unsharded element (row*n_kv_heads*head_dim + kv_head*head_dim + d) so that every sharding of
 * the same model sees the same cache.  For benchmarks and tests. */
int ligguf_cuda_attn_kv_synth(ligguf_attn* h, int layer0, int n_layers, int pos0, int n,
                              uint64_t seed, float scale);
/* Waits for all work the handle enqueued on its own stream (host-pointer calls). */
int ligguf_cuda_attn_sync(ligguf_attn* h);

/* ---- SARA all-gather over NVLink peer memory -------------------------------------------- */
/* The reference's SARA run reduces per-rank partials over TCP (cpp/ligguf_distrib.cpp:1025-1047).
 * Here every rank owns a KV-head slice and the per-head outputs are all-gathered.  These calls
 * set up a gather buffer of two slots of 64-bit words per rank (per slot: up to 8 merge groups of
 * [n_heads*head_dim] values plus their per-head max and sum, and a count word per head), shared
 * through CUDA IPC; decode_gather then stores this rank's results straight into every peer's
 * buffer from the decode kernel's epilogue, each value as one word (call epoch << 32 | 32 bits),
 * so a reader that sees the current epoch in a word has its value.  A head with one merge group
 * sends its output; a head split over several groups sends each group's (max, sum, o) and the
 * readers merge them.  gather_wait polls (bounded) until every word of the call carries its epoch
 * and writes the full fp32 vector to d_out.  The two calls alternate between the two slots. */
int ligguf_cuda_attn_gather_ipc_handle(ligguf_attn* h, void* handle_out /* 64 bytes */,
                                       size_t handle_size);
int ligguf_cuda_attn_gather_open(ligguf_attn* h, int nranks, int rank,
                                 const void* handles /* nranks * 64 bytes */,
                                 size_t handle_size);
int ligguf_cuda_attn_decode_gather_async(ligguf_attn* h, int layer, int pos, const float* d_q,
                                         const float* d_k, const float* d_v, void* stream);
int ligguf_cuda_attn_gather_wait_async(ligguf_attn* h, int layer, float* d_out, void* stream);

/* ---- BERT embedding attention ------------------------------------------------------------ */
/* Replaces the per-sequence loop of bert_embed() (fast/vdb.cpp:189-212): bidirectional
 * multi-head attention, no RoPE, no mask within a sequence.  Batched: `batch` sequences padded
 * to max_len, lens[b] valid tokens each (keys at or beyond lens[b] are masked out, padded query
 * rows are written as zeros).
 *   q,k,v,out [batch][max_len][n_heads*head_dim] fp32 (the reference's m_brt.q/k/v/ctx rows). */
typedef struct ligguf_bert_attn ligguf_bert_attn;
int ligguf_cuda_bert_init(int n_heads, int head_dim, int max_batch, int max_len, int device,
                          ligguf_bert_attn** out);
int ligguf_cuda_bert_free(ligguf_bert_attn* b);
int ligguf_cuda_bert_attn(ligguf_bert_attn* b, int batch, int max_len, const int* lens,
                          const float* q, const float* k, const float* v, float* out, int mode);
int ligguf_cuda_bert_attn_async(ligguf_bert_attn* b, int batch, int max_len, const int* d_lens,
                                const float* d_q, const float* d_k, const float* d_v,
                                float* d_out, int mode, void* stream);

/* ---- BERT attention without device allocation ------------------------------------------- */
/* No counterpart in the reference: an addition for callers that may not allocate device memory.
 * Such callers include hosts that route every device allocation through their own memory pool and
 * forbid libraries from calling cudaMalloc, and latency-critical loops where cudaMalloc's implicit
 * device-wide synchronisation and unbounded cost are not acceptable.
 *
 * Same computation as ligguf_cuda_bert_attn_async with LIGGUF_MODE_TC (bf16 operands on the
 * tcgen05 tensor cores, fp32 accumulation), but with no handle and no allocation: the bf16 copies
 * of q, k and v live in a fixed array inside the library, reserved on every GPU that loads it
 * (24.25 MiB + 256 B with the kernel's work order, held until the process exits).  Device pointers,
 * enqueued on `stream`, on the current device; layouts as ligguf_cuda_bert_attn.
 *   - Limit: batch*max_len*n_heads*head_dim <= LIGGUF_NOALLOC_MAX_ELEMS per tensor; larger calls
 *     return LIGGUF_ATTN_EINVAL without touching the GPU.
 *   - The first call on a device looks up the array's device address (cudaGetSymbolAddress); make
 *     that first call before any stream capture.  The address is looked up again when the device's
 *     context changes (after a cudaDeviceReset); a call must not be in flight across a reset.
 *   - Every call reuses the same array: calls whose work overlaps on the GPU (other streams, other
 *     host threads) race and corrupt each other; serialise them.  The kernel's error word is cleared
 *     at the start of each call.  A bounded in-kernel wait that gives up leaves `d_out` unwritten;
 *     the call itself has already returned, so ask ligguf_cuda_bert_attn_tc_noalloc_status. */
#define LIGGUF_NOALLOC_MAX_ELEMS (1 << 22)
int ligguf_cuda_bert_attn_tc_noalloc(int n_heads, int head_dim, int batch, int max_len, const int* d_lens,
                                     const float* d_q, const float* d_k, const float* d_v, float* d_out,
                                     void* stream);
/* Outcome of the no-allocation calls enqueued on the current device: waits for `stream` (a
 * cudaStream_t, NULL = legacy default), then returns LIGGUF_ATTN_ETIMEDOUT (and clears the word) if a
 * bounded wait in one of them gave up since the last call began, else 0.  Allocates nothing. */
int ligguf_cuda_bert_attn_tc_noalloc_status(void* stream);

/* ---- quantized projections (the QKV step of the forward pass) ---------------------------- */
/* Replaces quantize_q8_K + matmul3 at fast/ligguf_fast_qk.cpp:39-40 (fast/lil_math.cpp:352-385,
 * 827-899), and matmul / matmul2 (fast/lil_math.cpp:757-825) with one or two matrices: out[r] =
 * dot(row r of W, x) for weights in their GGUF block layout, with the activation quantized on the
 * device exactly as the reference quantizes it (Q8_K for the K-quants, Q8_0 for Q8_0 / Q1_0 / Q1_G,
 * fp32 for F32 / F16).  The integer block dot products and scale terms are exact; only the fp32 sum
 * over blocks runs in another order than the reference's AVX2 loops.
 * Weight types (gguf_type, fast/lil_gguf.h:26-44): 0 F32, 1 F16, 8 Q8_0, 10 Q2_K, 11 Q3_K, 12 Q4_K,
 * 13 Q5_K, 14 Q6_K, 40 Q1_0, 41 Q1_G.  Widths: a multiple of 32 (256 for K-quants), at most 16384,
 * and one row must fit a 32 KB stream stage (F32: at most 8192; init fails with
 * LIGGUF_ATTN_EUNSUPPORTED otherwise). */
typedef struct ligguf_qmat ligguf_qmat;
/* Bytes of one row of `n` elements of `type` (the reference's row_size), 0 if not a whole number of
 * blocks or an unknown type. */
size_t ligguf_cuda_qmat_row_bytes(int type, int n);
/* Copies a d x n weight matrix (d rows of ligguf_cuda_qmat_row_bytes(type, n) bytes, the GGUF tensor
 * as the engine mmaps it: wtensor::ptr / rsz, fast/lil_gguf.h:126-130) to HBM once. `rows` is host
 * memory, or device memory when rows_on_device is set. */
int ligguf_cuda_qmat_init(int type, int n, int d, const void* rows, int rows_on_device, int device,
                          ligguf_qmat** out);
/* Columns [col0, col0+ncols) of every row of such a matrix (whole blocks of the type): the SARA
 * shard's slice of attn_output, whose rank multiplies only its heads' columns
 * (matmul_partial_cols, cpp/ligguf_distrib.cpp:587-605,750).  The result is a d x ncols matrix. */
int ligguf_cuda_qmat_init_cols(int type, int n, int d, const void* rows, int col0, int ncols,
                               int rows_on_device, int device, ligguf_qmat** out);
int ligguf_cuda_qmat_free(ligguf_qmat* w);
/* matmul3 (w1, w2 non-NULL), matmul2 (w2 NULL) or matmul (w1, w2 NULL): device pointers, x [n],
 * out_i [d_i], enqueued on `stream` (a cudaStream_t; NULL = legacy default).  All matrices share n
 * and the device.  x is quantized once per call into a scratch owned by w0, so calls that share a
 * first matrix must be issued on one stream. */
int ligguf_cuda_matmul3_async(const ligguf_qmat* w0, const ligguf_qmat* w1, const ligguf_qmat* w2,
                              const float* d_x, float* d_out0, float* d_out1, float* d_out2,
                              void* stream);
/* Same with host pointers; returns when the outputs are written. */
int ligguf_cuda_matmul3(const ligguf_qmat* w0, const ligguf_qmat* w1, const ligguf_qmat* w2,
                        const float* x, float* out0, float* out1, float* out2);
/* Batched prompt projections: n_tok rows x [n_tok][n] -> out_i [n_tok][d_i], equal to n_tok calls of
 * the single-token form (the prompt loop of feed_text runs matmul3 once per token,
 * fast/ligguf_fast_qk.cpp:340-356); the weights stream from HBM once per group of up to 8 tokens. */
int ligguf_cuda_matmul3_batch_async(const ligguf_qmat* w0, const ligguf_qmat* w1, const ligguf_qmat* w2,
                                    const float* d_x, int n_tok, float* d_out0, float* d_out1,
                                    float* d_out2, void* stream);
int ligguf_cuda_matmul3_batch(const ligguf_qmat* w0, const ligguf_qmat* w1, const ligguf_qmat* w2,
                              const float* x, int n_tok, float* out0, float* out1, float* out2);
/* The activation quantizers on their own (device pointers), writing the reference's block layouts:
 * quantize_q8_K -> n/256 blocks {float d; int8 qs[256]; int16 bsums[16]} (292 bytes each), and
 * quantize_q8_0 -> n/32 blocks {fp16 d; int8 qs[32]} (34 bytes each); bit-identical to the
 * reference's results. */
int ligguf_cuda_quantize_q8_K_async(const float* d_x, int n, void* d_blocks, void* stream);
int ligguf_cuda_quantize_q8_0_async(const float* d_x, int n, void* d_blocks, void* stream);

/* ---- SARA attn_output projection + reduce over NVLink ------------------------------------- */
/* Replaces the tail of att_partial and the master's sum (cpp/ligguf_distrib.cpp:749-750,1025-1047):
 * every rank projects its heads' attention output through its columns of attn_output (a column slice,
 * ligguf_cuda_qmat_init_cols) and the partial rows are summed over the ranks.  Here the projection's
 * epilogue stores each partial row straight into every rank's reduce buffer over NVLink (CUDA IPC,
 * one 64-bit word (epoch << 32) | fp32 bits per row and rank, no fence, no flag), and a wait kernel on
 * every rank sums the ranks' rows in rank order (rank 0's, then += rank 1's, ... as the master does)
 * and adds the sum to the residual.  The reference sends the workers' partials over TCP quantized to
 * Q8_0 (:892-902); here they cross as fp32, so the sum does not carry that wire error.
 * Set-up: ligguf_cuda_reduce_init on every rank (rows = n_embed), exchange the 64-byte handles of
 * ligguf_cuda_reduce_ipc_handle (any side channel), ligguf_cuda_reduce_open with all of them in rank
 * order.  Per use: ligguf_cuda_matmul_reduce_async, then ligguf_cuda_reduce_wait_async on the same
 * stream (x_inout += sum, out = sum; either may be NULL).  Epochs live on the device, so the pair can
 * be captured in a CUDA graph.  Waits are bounded: ligguf_cuda_reduce_status reports a timeout. */
typedef struct ligguf_reduce ligguf_reduce;
int ligguf_cuda_reduce_init(int rows, int nranks, int rank, int device, ligguf_reduce** out);
int ligguf_cuda_reduce_free(ligguf_reduce* r);
int ligguf_cuda_reduce_ipc_handle(ligguf_reduce* r, void* handle_out /* 64 bytes */, size_t handle_size);
int ligguf_cuda_reduce_open(ligguf_reduce* r, const void* handles /* nranks * 64 bytes */,
                            size_t handle_size);
int ligguf_cuda_matmul_reduce_async(const ligguf_qmat* w, ligguf_reduce* r, const float* d_x,
                                    void* stream);
int ligguf_cuda_reduce_wait_async(ligguf_reduce* r, float* d_x_inout, float* d_out, void* stream);
int ligguf_cuda_reduce_status(ligguf_reduce* r, void* stream);

/* ---- seeded synthetic inputs ------------------------------------------------------------- */
/* Tensor ids of the synthetic generator's streams. */
#define LIGGUF_SYNTH_K 1
#define LIGGUF_SYNTH_V 2
#define LIGGUF_SYNTH_Q 3
#define LIGGUF_SYNTH_KNEW 4
#define LIGGUF_SYNTH_VNEW 5
#define LIGGUF_SYNTH_QGAMMA 6
#define LIGGUF_SYNTH_KGAMMA 7
/* dst[i] = (float)(a+b+c+d - 131070) * mul + add, rounded to dtype (LIGGUF_KV_*), where a..d are
 * the four 16-bit fields of splitmix64(splitmix64(seed ^ stream*0xD1B54A32D192ED03) + idx0 + i).
 * mul = scale / 37837.23 (computed in double, rounded to float) makes the values approximately
 * N(add, scale^2) (Irwin-Hall of 4 uniforms).  Integer arithmetic plus one fp32 multiply and
 * one add, so the host restatement reproduces it bit for bit. */
int ligguf_cuda_synth_fill(void* d_dst, int dtype, size_t n, uint64_t seed, uint64_t stream_id,
                           uint64_t idx0, float scale, float add, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* LIGGUF_CUDA_ATTN_H */
