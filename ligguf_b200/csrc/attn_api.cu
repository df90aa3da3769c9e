// attn_api.cu - the C ABI declared in include/ligguf_cuda_attn.h: handle life cycle, HBM-resident
// KV cache, argument checking, kernel dispatch and the host-pointer convenience calls.
//
// Nothing here falls back to the CPU: every compute entry point launches one of the CUDA kernels
// of this library or returns an error code.
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "ligguf_cuda_attn.h"
#include "api_util.h"
#include "common.cuh"
#include "decode.cuh"
#include "flash_simt.cuh"
#include "flash_tc.cuh"

namespace lgapi {
namespace {
thread_local std::string g_last_error;
}
int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}
const char* last_error() { return g_last_error.c_str(); }
}  // namespace lgapi

namespace {
using lgapi::DeviceGuard;
using lgapi::fail;

inline int ceil_div(long long a, long long b) { return static_cast<int>((a + b - 1) / b); }

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

size_t kv_elem_size(int kv_type) { return kv_type == LIGGUF_KV_F32 ? 4 : 2; }

CUtensorMapDataType kv_tmap_type(int kv_type) {
    return kv_type == LIGGUF_KV_F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
           : kv_type == LIGGUF_KV_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                      : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
}

// Raises the dynamic shared memory limit of `kernel` once per device.  `done` is the caller's
// per-instantiation flag array (function-pointer types are shared by all instantiations of a
// template kernel, so the flags cannot live here).
template <typename K>
cudaError_t ensure_smem_attr(K kernel, int device, size_t bytes, bool* done) {
    if (device >= 0 && device < 64 && done[device]) return cudaSuccess;
    const cudaError_t e =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
    if (e == cudaSuccess && device >= 0 && device < 64) done[device] = true;
    return e;
}

// ---------------------------------------------------------------------------- synth kernels
template <typename T>
__global__ void synth_fill_kernel(T* dst, size_t n, uint64_t base, uint64_t idx0, float mul, float add) {
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
        dst[i] = lg::KvTraits<T>::from_float(lg::synth_value(base, idx0 + i, mul, add));
}

template <typename T>
__global__ void kv_synth_kernel(T* layer_base, int kv_dim, int kv_dim_full, int kv_off, int pos0, int n,
                                uint64_t base, float mul) {
    const size_t total = size_t(n) * kv_dim;
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
        const int rr = static_cast<int>(i / kv_dim), c = static_cast<int>(i % kv_dim);
        const size_t t = size_t(pos0) + rr;
        const uint64_t idx = uint64_t(t) * uint64_t(kv_dim_full) + uint64_t(kv_off + c);
        layer_base[t * kv_dim + c] = lg::KvTraits<T>::from_float(lg::synth_value(base, idx, mul, 0.f));
    }
}

float synth_mul(float scale) { return static_cast<float>(static_cast<double>(scale) / lg::kSynthSd); }

// ---------------------------------------------------------------------------- gather wait
// Gather wait: one thread per element polls its 64-bit words in this rank's gather slot until they
// carry the call's epoch (bounded), then writes the fp32 value to `out`.  The head's count word says
// what the shard stored: 1, the normalised output in group 0; G > 1, G first-level merge groups
// (o unnormalised, m, l), which are merged here as the shard's second merge level would have (weights
// e^(m_g - M), out = sum w_g o_g / sum w_g l_g).  All of an element's words are loaded before any is
// checked, so the polls overlap.  The epoch is gstate[0] + 1 (gstate[0] = the last completed call's
// epoch, advanced here by the last block to finish, gstate[1] counting the finished blocks), the slot
// is epoch & 1: nothing of a call is decided on the host, so a captured CUDA graph replays correctly.
// Launched as a programmatic dependent of the decode kernel, it starts while the decode still runs;
// it reads nothing the decode writes other than these self-validating words, so it never waits for
// the decode grid itself (the decode reads gstate[0] only after this kernel's predecessor completed,
// and the next decode only after this one completed).
__device__ __forceinline__ unsigned long long ld_word(const unsigned long long* p) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

__global__ void __launch_bounds__(256) gather_wait_kernel(const unsigned long long* words_base, int* gstate,
                                                          float* out, int heads, int d, int* err) {
    constexpr int G = lg::kGatherGroups;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int epoch = __ldcg(gstate) + 1;
    const size_t vec = size_t(heads) * d;
    const unsigned long long* slot = words_base + size_t(epoch & 1) * lg::gather_slot_words(heads, d);
    const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < vec) {
        const int h = static_cast<int>(i / d);
        const uint64_t deadline = lg::globaltimer_ns() + lg::kWaitLimitNs;
        const uint32_t want = static_cast<uint32_t>(epoch);
        auto cur = [want](unsigned long long w) { return static_cast<uint32_t>(w >> 32) == want; };
        auto val = [](unsigned long long w) { return __uint_as_float(static_cast<uint32_t>(w)); };
        const unsigned long long* pc = slot + lg::gather_cnt_off(heads, d) + h;
        const unsigned long long* pm = slot + lg::gather_m_off(heads, d) + h;
        const unsigned long long* pl = slot + lg::gather_l_off(heads, d) + h;
        unsigned long long wc = ld_word(pc), wo[G], wm[G], wl[G];
#pragma unroll
        for (int g = 0; g < G; ++g) wo[g] = wm[g] = wl[g] = 0ull;
        uint32_t spins = 0;
        int ng = 0;  // groups of this element, once its count word is current
        bool ok = true;
        while (true) {
            bool done = false;
            if (!ng && cur(wc)) {
                ng = static_cast<int>(static_cast<uint32_t>(wc));
                if (ng < 1 || ng > G) {  // not a count this library stores
                    *reinterpret_cast<volatile int*>(err) = lg::KERR_TIMEOUT_PEER;
                    ok = false;
                    break;
                }
#pragma unroll
                for (int g = 0; g < G; ++g)
                    if (g < ng) {
                        wo[g] = ld_word(slot + g * vec + i);
                        if (ng > 1) {
                            wm[g] = ld_word(pm + g * heads);
                            wl[g] = ld_word(pl + g * heads);
                        }
                    }
            }
            if (ng) {
                done = true;
#pragma unroll
                for (int g = 0; g < G; ++g)
                    if (g < ng) {
                        if (!cur(wo[g])) {
                            done = false;
                            wo[g] = ld_word(slot + g * vec + i);
                        }
                        if (ng > 1 && !cur(wm[g])) {
                            done = false;
                            wm[g] = ld_word(pm + g * heads);
                        }
                        if (ng > 1 && !cur(wl[g])) {
                            done = false;
                            wl[g] = ld_word(pl + g * heads);
                        }
                    }
            } else {
                wc = ld_word(pc);
            }
            if (done) break;
            if ((++spins & 63u) == 0u && lg::globaltimer_ns() > deadline) {
                *reinterpret_cast<volatile int*>(err) = lg::KERR_TIMEOUT_PEER;
                ok = false;
                break;
            }
        }
        if (ok) {
            if (ng == 1) {
                out[i] = val(wo[0]);
            } else {
                float M = -INFINITY;
#pragma unroll
                for (int g = 0; g < G; ++g)
                    if (g < ng) M = fmaxf(M, val(wm[g]));
                float L = 0.f, O = 0.f;
#pragma unroll
                for (int g = 0; g < G; ++g)
                    if (g < ng) {
                        const float mv = val(wm[g]);
                        const float w = mv == -INFINITY ? 0.f : expf(mv - M);
                        L = fmaf(val(wl[g]), w, L);
                        O = fmaf(val(wo[g]), w, O);
                    }
                out[i] = O / L;
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(&gstate[1], 1) == static_cast<int>(gridDim.x) - 1) {
        gstate[1] = 0;
        gstate[0] = epoch;  // read by the next call's kernels, which start after this grid completes
    }
}

}  // namespace

// ============================================================================== handle
struct ligguf_attn {
    ligguf_attn_cfg cfg{};
    int nrep = 0, q_headn = 0, kv_dim = 0, kv_dim_full = 0, rope_pairs = 0, num_sms = 0;
    size_t es = 0, layer_elems = 0;
    void* kc = nullptr;
    void* vc = nullptr;
    float* freq = nullptr;
    float* qg = nullptr;  // [n_layers][D]
    float* kg = nullptr;
    std::vector<uint8_t> norm_set;
    // Cache rows written by the most recent call that writes the cache (possibly still running when
    // the next decode starts): layers [wr_l0, wr_l1), rows from wr_row0 up.  A decode may load rows
    // below it before its predecessor grid completes.
    int wr_l0 = 0, wr_l1 = 0, wr_row0 = 0;
    float* part = nullptr;
    float* gpart = nullptr;
    int* counters = nullptr;
    int* h_err = nullptr;  // mapped pinned word the kernels write on failure
    int* d_err = nullptr;
    cudaStream_t stream = nullptr;
    float* d_stage = nullptr;  // device staging for the host-pointer calls
    size_t stage_floats = 0;
    float* h_stage = nullptr;  // pinned, mapped host staging for the host-pointer decode
    float* h_stage_dev = nullptr;  // its device address
    size_t h_stage_floats = 0;
    float* qf = nullptr;  // prefill fp32 q rows
    size_t qf_floats = 0;
    __nv_bfloat16* qb = nullptr;  // prefill bf16 q rows
    size_t qb_elems = 0;
    // bf16 shadows of the K/V cache for the tensor-core prefill, per layer [n_context][kv_dim],
    // allocated at a layer's first tensor-core prefill; d_wm[layer]: shadow rows [0, d_wm[layer])
    // match the cache (the decode kernel, the SIMT prefill and the host writes lower it; the
    // tensor-core prefill converts only the rows between it and pos0, then raises it).
    std::vector<__nv_bfloat16*> kb, vb;
    int* d_wm = nullptr;
    alignas(64) CUtensorMap tm_k;
    alignas(64) CUtensorMap tm_v;
    // SARA gather over CUDA IPC
    unsigned long long* gbuf = nullptr;  // [2][gather_slot_words] gather words: (epoch << 32) | 32 bits
    size_t gbuf_bytes = 0;
    int g_nranks = 0, g_rank = -1;
    bool g_pending = false;   // a gathered decode was enqueued and its wait not yet
    int* d_gstate = nullptr;  // device: [0] last completed gather epoch, [1] finished wait blocks
    std::vector<void*> g_opened;
    unsigned long long** d_peer_ll = nullptr;  // [2][nranks]: slot s of every rank's gather buffer
};

struct ligguf_bert_attn {
    int n_heads = 0, head_dim = 0, max_batch = 0, max_len = 0, device = 0;
    int* d_lens = nullptr;
    float* d_buf = nullptr;  // q, k, v, out staging for the host-pointer call
    __nv_bfloat16* bf = nullptr;  // bf16 q, k, v for the tensor-core path
    int* d_order = nullptr;       // the tensor-core kernel's work order (bert_item_order)
    int* h_err = nullptr;
    int* d_err = nullptr;
    cudaStream_t stream = nullptr;
};

namespace {

int check_err_word(int* h_err, int* counters, size_t n_counters) {
    if (h_err && *reinterpret_cast<volatile int*>(h_err)) {
        const int code = *h_err;
        *reinterpret_cast<volatile int*>(h_err) = 0;
        if (counters) cudaMemset(counters, 0, n_counters * sizeof(int));
        return fail(LIGGUF_ATTN_ETIMEDOUT, "a bounded in-kernel wait gave up (kernel error code %d)", code);
    }
    return LIGGUF_ATTN_OK;
}

int make_cache_tmap(CUtensorMap* m, void* base, const ligguf_attn* h, int tile_rows) {
    auto enc = tensor_map_encoder();
    if (!enc) return fail(LIGGUF_ATTN_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const int D = h->cfg.head_dim;
    const int kvh = h->kv_dim / D;
    cuuint64_t dims[3] = {cuuint64_t(D), cuuint64_t(kvh),
                          cuuint64_t(h->cfg.n_layers) * cuuint64_t(h->cfg.n_context)};
    cuuint64_t strides[2] = {cuuint64_t(D) * h->es, cuuint64_t(h->kv_dim) * h->es};
    cuuint32_t box[3] = {cuuint32_t(D), 1u, cuuint32_t(tile_rows)};
    cuuint32_t estr[3] = {1u, 1u, 1u};
    const CUresult r = enc(m, kv_tmap_type(h->cfg.kv_type), 3, base, dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(LIGGUF_ATTN_ECUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
    return LIGGUF_ATTN_OK;
}

int decode_tile_rows(int kv_type, int D) { return lg::kDecodeTileBytes / (D * int(kv_elem_size(kv_type))); }

template <typename KV, int D, int NREP>
int launch_decode_t(ligguf_attn* h, const lg::DecodeArgs& a, cudaStream_t st) {
    using Sm = lg::DecodeSmem<KV, D, NREP>;
    auto kern = lg::decode_kernel<KV, D, NREP>;
    static bool attr_done[64] = {};
    LG_CUDA(ensure_smem_attr(kern, h->cfg.device, Sm::kTotal, attr_done));
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(h->kv_dim / D, a.n_split, 1);
    lc.blockDim = dim3(lg::kDecodeThreads, 1, 1);
    lc.dynamicSmemBytes = Sm::kTotal;
    lc.stream = st;
    // Programmatic dependent launch: the kernel may start while the previous kernel of the stream
    // finishes; it waits for that grid (griddepcontrol.wait) before its first global read.
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    LG_CUDA(cudaLaunchKernelEx(&lc, kern, h->tm_k, h->tm_v, a));
    return LIGGUF_ATTN_OK;
}

template <typename KV, int D>
int launch_decode_d(ligguf_attn* h, const lg::DecodeArgs& a, cudaStream_t st) {
    switch (h->nrep) {
        case 1: return launch_decode_t<KV, D, 1>(h, a, st);
        case 2: return launch_decode_t<KV, D, 2>(h, a, st);
        case 4: return launch_decode_t<KV, D, 4>(h, a, st);
        case 8: return launch_decode_t<KV, D, 8>(h, a, st);
        default: return fail(LIGGUF_ATTN_EUNSUPPORTED, "nrep %d has no decode kernel (1, 2, 4, 8)", h->nrep);
    }
}

template <typename KV>
int launch_decode_k(ligguf_attn* h, const lg::DecodeArgs& a, cudaStream_t st) {
    if (h->cfg.head_dim == 64) return launch_decode_d<KV, 64>(h, a, st);
    if (h->cfg.head_dim == 128) return launch_decode_d<KV, 128>(h, a, st);
    return fail(LIGGUF_ATTN_EUNSUPPORTED, "head_dim %d has no decode kernel", h->cfg.head_dim);
}

// Blocks of the decode kernel resident per SM (its __launch_bounds__ minimum).
int decode_blocks_per_sm(int kv_type, int nrep) { return nrep * (kv_type == LIGGUF_KV_F32 ? 4 : 8) > 32 ? 1 : 2; }

void note_cache_write(ligguf_attn* h, int layer0, int n_layers, int row0) {
    h->wr_l0 = layer0;
    h->wr_l1 = layer0 + n_layers;
    h->wr_row0 = row0;
}

// A host-side write of cache rows from row0 up in layers [layer0, +n_layers): the bf16 shadows of
// those rows are stale.  On the handle's stream, then waited for (the callers are synchronous).
int lower_shadow_marks(ligguf_attn* h, int layer0, int n_layers, int row0) {
    lg::shadow_lower_kernel<<<1, 256, 0, h->stream>>>(h->d_wm + layer0, n_layers, row0);
    LG_CUDA(cudaGetLastError());
    LG_CUDA(cudaStreamSynchronize(h->stream));
    return LIGGUF_ATTN_OK;
}

int decode_enqueue(ligguf_attn* h, int layer, int pos, const float* dq, const float* dk, const float* dv,
                   float* dout, cudaStream_t st, bool gather) {
    const ligguf_attn_cfg& c = h->cfg;
    if (layer < 0 || layer >= c.n_layers) return fail(LIGGUF_ATTN_EINVAL, "layer %d out of range", layer);
    if (pos < 0 || pos >= c.n_context)
        return fail(LIGGUF_ATTN_EINVAL, "pos %d out of range [0, %d)", pos, c.n_context);
    if (!dq || !dk || !dv || (!dout && !gather)) return fail(LIGGUF_ATTN_EINVAL, "null tensor pointer");
    if (c.qk_norm && !h->norm_set[layer])
        return fail(LIGGUF_ATTN_ESTATE, "QK-norm weights of layer %d were not set", layer);
    const int D = c.head_dim;
    lg::DecodeArgs a = {};
    a.q = dq;
    a.k = dk;
    a.v = dv;
    a.qg = c.qk_norm ? h->qg + size_t(layer) * D : nullptr;
    a.kg = c.qk_norm ? h->kg + size_t(layer) * D : nullptr;
    a.freq = h->freq;
    a.kc = static_cast<char*>(h->kc) + size_t(layer) * h->layer_elems * h->es;
    a.vc = static_cast<char*>(h->vc) + size_t(layer) * h->layer_elems * h->es;
    a.out = dout;
    a.part = h->part;
    a.gpart = h->gpart;
    a.counters = h->counters;
    a.err = h->d_err;
    a.shadow_wm = h->d_wm + layer;
    a.row0 = layer * c.n_context;
    a.pos = pos;
    const int tp = decode_tile_rows(c.kv_type, D);
    a.n_tiles = ceil_div(pos, tp);
    const int kvh = h->kv_dim / D;
    // One resident wave: blocks_per_sm * SMs CTAs shared by the KV heads.  Each CTA starts on one
    // static chunk and then grabs chunks of its head dynamically: single tiles up to ~48 tiles per
    // CTA (finish times then differ by about one tile), larger chunks beyond.
    const int want = std::max(1, decode_blocks_per_sm(c.kv_type, h->nrep) * h->num_sms / kvh);
    a.n_split = std::max(1, std::min(want, a.n_tiles));
    // The two-level merge takes groups of decode_merge_group partials (what one copy into the tile
    // ring holds), then the group results in one more copy: at most that many groups, and at most
    // kDecodeMaxGroups counters per head.
    const int mg = lg::decode_merge_group(h->nrep, D);
    a.n_split = std::min(a.n_split, std::min(lg::kDecodeMaxSplit, mg * std::min(lg::kDecodeMaxGroups, mg)));
    // Few tiles per CTA (short contexts, one KV head per GPU): static contiguous chunks of equal size
    // cover every tile; a CTA then requests its whole chunk (up to the ring's depth) before the
    // previous kernel completes, and no CTA waits on a grab.  More tiles per CTA: a static first
    // chunk, then dynamic grabs, single tiles up to ~48 tiles per CTA, larger chunks beyond.
    const int per_cta = ceil_div(a.n_tiles, a.n_split);
    if (per_cta <= lg::kDecodeStaticMaxTiles) {
        a.chunk = std::max(1, per_cta);
        a.n_split = ceil_div(a.n_tiles, a.chunk);
        a.dynamic = 0;
    } else {
        a.chunk = std::max(1, a.n_tiles / (a.n_split * 48));
        a.dynamic = a.n_split > 1;
    }
    a.n_split = std::max(1, a.n_split);
    // First-level merge groups: as large as one copy into the ring allows; a gathered decode spreads
    // its splits over up to kGatherGroups smaller groups instead, whose results the gather wait merges.
    a.merge_group = gather ? std::min(mg, std::max(1, ceil_div(a.n_split, lg::kGatherGroups))) : mg;
    a.chunk_ctr = h->counters + kvh;
    a.kv_dim = h->kv_dim;
    a.rope_pairs = h->rope_pairs;
    a.qk_norm = c.qk_norm;
    a.scale_div = c.scale_mode == LIGGUF_SCALE_DIV;
    a.scale = a.scale_div ? sqrtf(static_cast<float>(D)) : 1.0f / sqrtf(static_cast<float>(D));
    a.eps = c.rms_epsilon;
    a.kv_head0 = c.kv_head0;
    a.pre_rows = (layer >= h->wr_l0 && layer < h->wr_l1) ? std::min(pos, h->wr_row0) : pos;
    note_cache_write(h, layer, 1, pos);
    if (gather) {
        a.peer_ll = h->d_peer_ll;
        a.nranks = h->g_nranks;
        a.rank = h->g_rank;
        a.g_heads = c.n_heads;
        a.q_off = c.kv_head0 * h->nrep * D;
        a.epoch = h->d_gstate;
    }
    switch (c.kv_type) {
        case LIGGUF_KV_F32: return launch_decode_k<float>(h, a, st);
        case LIGGUF_KV_F16: return launch_decode_k<__half>(h, a, st);
        default: return launch_decode_k<__nv_bfloat16>(h, a, st);
    }
}

// ---------------------------------------------------------------------------- flash launches
template <typename KV, int D>
int launch_flash_simt_t(const lg::FlashArgs& f, dim3 grid, cudaStream_t st, int device) {
    auto kern = lg::flash_simt_kernel<KV, D>;
    static bool attr_done[64] = {};
    LG_CUDA(ensure_smem_attr(kern, device, lg::FlashSimtSmem<D>::kBytes, attr_done));
    kern<<<grid, lg::kFlashThreads, lg::FlashSimtSmem<D>::kBytes, st>>>(f);
    LG_CUDA(cudaGetLastError());
    return LIGGUF_ATTN_OK;
}

template <typename KV>
int launch_flash_simt(const lg::FlashArgs& f, int D, dim3 grid, cudaStream_t st, int device) {
    if (D == 64) return launch_flash_simt_t<KV, 64>(f, grid, st, device);
    if (D == 128) return launch_flash_simt_t<KV, 128>(f, grid, st, device);
    return fail(LIGGUF_ATTN_EUNSUPPORTED, "head_dim %d has no SIMT attention kernel", D);
}

template <typename KV, int D>
int launch_prep_t(const lg::PrepArgs& p, cudaStream_t st) {
    // One block per token; the token's q, k, v rows in dynamic shared memory.
    const int smem = (p.q_headn + 2 * p.kv_headn) * D * 4;
    auto kern = lg::prefill_prep_kernel<KV, D>;
    if (smem > 48 * 1024) LG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kern<<<p.n, lg::kPrepWarps * 32, smem, st>>>(p);
    LG_CUDA(cudaGetLastError());
    return LIGGUF_ATTN_OK;
}

template <typename KV>
int launch_prep(const lg::PrepArgs& p, int D, cudaStream_t st) {
    if (D == 64) return launch_prep_t<KV, 64>(p, st);
    if (D == 128) return launch_prep_t<KV, 128>(p, st);
    return fail(LIGGUF_ATTN_EUNSUPPORTED, "head_dim %d has no prefill kernel", D);
}

template <typename T>
int grow(T** p, size_t* cap, size_t need) {
    if (*cap >= need) return LIGGUF_ATTN_OK;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    if (cudaMalloc(reinterpret_cast<void**>(p), need * sizeof(T)) != cudaSuccess)
        return fail(LIGGUF_ATTN_ENOMEM, "cudaMalloc of %zu bytes failed", need * sizeof(T));
    *cap = need;
    return LIGGUF_ATTN_OK;
}

// ---------------------------------------------------------------------------- tensor-core launch
int make_bf16_tmap(CUtensorMap* m, const void* base, int D, int heads, int rows, int box_rows) {
    auto enc = tensor_map_encoder();
    if (!enc) return fail(LIGGUF_ATTN_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
    cuuint64_t dims[3] = {cuuint64_t(D), cuuint64_t(heads), cuuint64_t(rows)};
    cuuint64_t strides[2] = {cuuint64_t(D) * 2, cuuint64_t(heads) * D * 2};
    cuuint32_t box[3] = {64u, 1u, cuuint32_t(box_rows)};
    cuuint32_t estr[3] = {1u, 1u, 1u};
    const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(LIGGUF_ATTN_ECUDA, "cuTensorMapEncodeTiled (bf16 operand) failed (%d)", int(r));
    return LIGGUF_ATTN_OK;
}

template <int D>
int launch_flash_tc_t(const lg::TcArgs& t, cudaStream_t st, int device) {
    alignas(64) CUtensorMap tq, tk, tv;
    int rc;
    if ((rc = make_bf16_tmap(&tq, t.q, D, t.q_heads, t.q_rows, lg::kTcRows))) return rc;
    if ((rc = make_bf16_tmap(&tk, t.k, D, t.kv_heads, t.kv_rows, lg::kTcKeys))) return rc;
    if ((rc = make_bf16_tmap(&tv, t.v, D, t.kv_heads, t.kv_rows, lg::kTcKeys))) return rc;
    auto kern = lg::flash_tc_kernel<D>;
    static bool attr_done[64] = {};
    LG_CUDA(ensure_smem_attr(kern, device, lg::TcSmem<D>::kTotal, attr_done));
    // Persistent grid: as many CTAs as are resident at once (one per SM: the runtime places one CTA
    // of a tcgen05 kernel per SM), each walking its share of the (head, query tile, batch entry) items.
    static int resident[64] = {};
    int slots = device >= 0 && device < 64 ? resident[device] : 0;
    if (slots == 0) {
        // The warpgroups' register shares (setmaxnreg) come out of the registers the CTA launched
        // with; a smaller launch count would leave the softmax warpgroup's increase waiting forever.
        cudaFuncAttributes fa{};
        LG_CUDA(cudaFuncGetAttributes(&fa, kern));
        constexpr int need = lg::kTcRegsIssue + 2 * lg::kTcRegsSoftmax + lg::kTcRegsEpilogue;
        if (fa.numRegs * 4 < need)
            return fail(LIGGUF_ATTN_ECUDA, "tensor-core attention kernel built with %d registers per thread, %d needed",
                        fa.numRegs, (need + 3) / 4);
        int sms = 0, per_sm = 0;
        LG_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
        LG_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, lg::kTcThreads, lg::TcSmem<D>::kTotal));
        if (per_sm < 1) return fail(LIGGUF_ATTN_ECUDA, "the tensor-core attention kernel does not fit on an SM");
        slots = sms * per_sm;
        if (device >= 0 && device < 64) resident[device] = slots;
    }
    const int n_items = t.q_heads * ((t.q_seq + lg::kTcRows - 1) / lg::kTcRows) * t.batch;
    if (n_items <= 0) return LIGGUF_ATTN_OK;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(std::min(n_items, slots), 1, 1);
    lc.blockDim = dim3(lg::kTcThreads, 1, 1);
    lc.dynamicSmemBytes = lg::TcSmem<D>::kTotal;
    lc.stream = st;
    // Programmatic dependent of the operand kernel launched just before it (prefill_prep_kernel or
    // bert_to_bf16_kernel, which trigger at entry): the CTAs' set-up overlaps that grid's tail, and
    // the kernel waits for it (griddepcontrol.wait) before any global access.
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    LG_CUDA(cudaLaunchKernelEx(&lc, kern, tq, tk, tv, t));
    return LIGGUF_ATTN_OK;
}

int launch_flash_tc(const lg::TcArgs& t, int D, cudaStream_t st, int device) {
    if (D == 64) return launch_flash_tc_t<64>(t, st, device);
    if (D == 128) return launch_flash_tc_t<128>(t, st, device);
    return fail(LIGGUF_ATTN_EUNSUPPORTED, "head_dim %d has no tensor-core attention kernel", D);
}

int prefill_enqueue(ligguf_attn* h, int layer, int pos0, int n, const float* dq, const float* dk, const float* dv,
                    float* dout, int mode, cudaStream_t st) {
    const ligguf_attn_cfg& c = h->cfg;
    if (layer < 0 || layer >= c.n_layers) return fail(LIGGUF_ATTN_EINVAL, "layer %d out of range", layer);
    if (n < 1 || pos0 < 0 || pos0 + n > c.n_context)
        return fail(LIGGUF_ATTN_EINVAL, "positions [%d, %d) outside [0, %d)", pos0, pos0 + n, c.n_context);
    if (!dq || !dk || !dv || !dout) return fail(LIGGUF_ATTN_EINVAL, "null tensor pointer");
    if ((reinterpret_cast<uintptr_t>(dq) | reinterpret_cast<uintptr_t>(dk) | reinterpret_cast<uintptr_t>(dv)) & 15)
        return fail(LIGGUF_ATTN_EINVAL, "q, k and v must be 16-byte aligned");
    if (mode != LIGGUF_MODE_SIMT && mode != LIGGUF_MODE_TC) return fail(LIGGUF_ATTN_EINVAL, "mode %d", mode);
    if (c.qk_norm && !h->norm_set[layer])
        return fail(LIGGUF_ATTN_ESTATE, "QK-norm weights of layer %d were not set", layer);
    const int D = c.head_dim;
    const size_t qn = size_t(n) * h->q_headn * D;
    note_cache_write(h, layer, 1, pos0);
    lg::PrepArgs p = {};
    p.q = dq;
    p.k = dk;
    p.v = dv;
    p.qg = c.qk_norm ? h->qg + size_t(layer) * D : nullptr;
    p.kg = c.qk_norm ? h->kg + size_t(layer) * D : nullptr;
    p.freq = h->freq;
    p.kc = static_cast<char*>(h->kc) + size_t(layer) * h->layer_elems * h->es;
    p.vc = static_cast<char*>(h->vc) + size_t(layer) * h->layer_elems * h->es;
    p.n = n;
    p.pos0 = pos0;
    p.q_headn = h->q_headn;
    p.kv_headn = h->kv_dim / D;
    p.kv_dim = h->kv_dim;
    p.rope_pairs = h->rope_pairs;
    p.qk_norm = c.qk_norm;
    p.eps = c.rms_epsilon;
    p.wm = h->d_wm + layer;
    p.err = h->d_err;
    const bool div = c.scale_mode == LIGGUF_SCALE_DIV;
    const float scale = div ? sqrtf(static_cast<float>(D)) : 1.0f / sqrtf(static_cast<float>(D));

    if (mode == LIGGUF_MODE_SIMT) {
        int rc = grow(&h->qf, &h->qf_floats, qn);
        if (rc) return rc;
        p.qf = h->qf;
        switch (c.kv_type) {
            case LIGGUF_KV_F32: rc = launch_prep<float>(p, D, st); break;
            case LIGGUF_KV_F16: rc = launch_prep<__half>(p, D, st); break;
            default: rc = launch_prep<__nv_bfloat16>(p, D, st); break;
        }
        if (rc) return rc;
        lg::FlashArgs f = {};
        f.q = h->qf;
        f.q_row = h->q_headn * D;
        f.k = p.kc;
        f.v = p.vc;
        f.kv_row = h->kv_dim;
        f.out = dout;
        f.o_row = h->q_headn * D;
        f.n_q = n;
        f.kv_len = pos0 + n;
        f.causal = 1;
        f.q_pos0 = pos0;
        f.nrep = h->nrep;
        f.scale_div = div;
        f.scale = scale;
        const dim3 grid(ceil_div(n, lg::kFlashBQ), h->q_headn, 1);
        switch (c.kv_type) {
            case LIGGUF_KV_F32: return launch_flash_simt<float>(f, D, grid, st, c.device);
            case LIGGUF_KV_F16: return launch_flash_simt<__half>(f, D, grid, st, c.device);
            default: return launch_flash_simt<__nv_bfloat16>(f, D, grid, st, c.device);
        }
    }

    // Tensor-core path: bf16 q rows, this layer's bf16 K/V shadow rows [0, pos0+n).
    int rc = grow(&h->qb, &h->qb_elems, qn);
    if (rc) return rc;
    if (!h->kb[layer]) {
        const size_t bytes = size_t(c.n_context) * h->kv_dim * sizeof(__nv_bfloat16);
        if (cudaMalloc(&h->kb[layer], bytes) != cudaSuccess || cudaMalloc(&h->vb[layer], bytes) != cudaSuccess)
            return fail(LIGGUF_ATTN_ENOMEM, "bf16 K/V shadow allocation failed");
    }
    p.qb = h->qb;
    p.kb = h->kb[layer];
    p.vb = h->vb[layer];
    if (pos0 > 0) {  // cache rows written since the shadows last matched -> bf16
        const int blocks = std::min(4 * h->num_sms, std::max(1, ceil_div(size_t(pos0) * h->kv_dim, 256)));
        switch (c.kv_type) {
            case LIGGUF_KV_F32:
                lg::shadow_sync_kernel<float><<<blocks, 256, 0, st>>>(static_cast<const float*>(p.kc),
                                                                      static_cast<const float*>(p.vc), p.kb, p.vb,
                                                                      h->kv_dim, p.wm, pos0);
                break;
            case LIGGUF_KV_F16:
                lg::shadow_sync_kernel<__half><<<blocks, 256, 0, st>>>(static_cast<const __half*>(p.kc),
                                                                       static_cast<const __half*>(p.vc), p.kb, p.vb,
                                                                       h->kv_dim, p.wm, pos0);
                break;
            default:
                lg::shadow_sync_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
                    static_cast<const __nv_bfloat16*>(p.kc), static_cast<const __nv_bfloat16*>(p.vc), p.kb, p.vb,
                    h->kv_dim, p.wm, pos0);
                break;
        }
        LG_CUDA(cudaGetLastError());
    }
    switch (c.kv_type) {
        case LIGGUF_KV_F32: rc = launch_prep<float>(p, D, st); break;
        case LIGGUF_KV_F16: rc = launch_prep<__half>(p, D, st); break;
        default: rc = launch_prep<__nv_bfloat16>(p, D, st); break;
    }
    if (rc) return rc;
    lg::TcArgs t = {};
    t.q = h->qb;
    t.k = p.kb;
    t.v = p.vb;
    t.out = dout;
    t.q_rows = n;
    t.q_heads = h->q_headn;
    t.kv_rows = pos0 + n;
    t.kv_heads = h->kv_dim / D;
    t.batch = 1;
    t.q_seq = n;
    t.kv_seq = pos0 + n;
    t.lens = nullptr;
    t.causal = 1;
    t.q_pos0 = pos0;
    t.nrep = h->nrep;
    t.scale_log2 = (div ? 1.0f / sqrtf(static_cast<float>(D)) : scale) * 1.4426950408889634f;
    t.err = h->d_err;
    return launch_flash_tc(t, D, st, c.device);
}

}  // namespace

// ============================================================================== no-allocation scratch
// Scratch of ligguf_cuda_bert_attn_tc_noalloc, reserved in every GPU that loads this library for as
// long as the process lives: the bf16 copies of q, k and v (LIGGUF_NOALLOC_MAX_ELEMS elements
// each, 8 MiB apiece), 256 bytes holding the kernel's error word, then the tensor-core kernel's work
// order (one int per work item: n_heads * ceil(max_len / 128) * batch <= elements / 64, since
// head_dim >= 64).  Host code must not hand the symbol itself to a kernel (on the host it is only a
// stand-in for the device array); the device address comes from cudaGetSymbolAddress, once per
// device.
constexpr size_t kNoallocOperandBytes = size_t(LIGGUF_NOALLOC_MAX_ELEMS) * sizeof(__nv_bfloat16);
constexpr size_t kNoallocOrderInts = size_t(LIGGUF_NOALLOC_MAX_ELEMS) / 64;
constexpr size_t kNoallocBytes = 3 * kNoallocOperandBytes + 256 + kNoallocOrderInts * sizeof(int);
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocBytes];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_addr[64] = {};
CUcontext g_noalloc_ctx[64] = {};  // the context each cached address belongs to

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CtxGetCurrentFn ctx_get_current() {
    static CtxGetCurrentFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<CtxGetCurrentFn>(p);
    }
    return fn;
}

CUcontext current_ctx() {
    CUcontext c = nullptr;
    if (auto f = ctx_get_current()) {
        if (f(&c) != CUDA_SUCCESS) c = nullptr;
    }
    return c;
}

// Device address of g_noalloc_scratch on the current device.  Looked up on the first call there, and
// again whenever the current context is not the one the cached address came from (after a
// cudaDeviceReset the module is loaded anew and the old address is stale).
int noalloc_scratch(int device, unsigned char** out) {
    if (device < 0 || device >= 64) return fail(LIGGUF_ATTN_EINVAL, "device %d", device);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[device] || current_ctx() != g_noalloc_ctx[device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            (void)cudaGetLastError();
            return fail(LIGGUF_ATTN_ECUDA, "cudaGetSymbolAddress of the no-allocation scratch failed: %s",
                        cudaGetErrorString(e));
        }
        g_noalloc_addr[device] = p;
        g_noalloc_ctx[device] = current_ctx();  // the lookup made the device's context current
    }
    *out = static_cast<unsigned char*>(g_noalloc_addr[device]);
    return LIGGUF_ATTN_OK;
}
}  // namespace

// ============================================================================== C ABI
extern "C" {

const char* ligguf_cuda_attn_strerror(int status) {
    switch (status) {
        case LIGGUF_ATTN_OK: return "ok";
        case LIGGUF_ATTN_EINVAL: return "invalid argument";
        case LIGGUF_ATTN_ECUDA: return "CUDA error";
        case LIGGUF_ATTN_ENOMEM: return "out of memory";
        case LIGGUF_ATTN_ETIMEDOUT: return "in-kernel wait timed out";
        case LIGGUF_ATTN_EUNSUPPORTED: return "unsupported shape or type";
        case LIGGUF_ATTN_ESTATE: return "invalid state for this call";
        default: return "unknown status";
    }
}

const char* ligguf_cuda_attn_last_error(void) { return lgapi::last_error(); }

int ligguf_cuda_attn_free(ligguf_attn* h) {
    if (!h) return LIGGUF_ATTN_OK;
    DeviceGuard dg(h->cfg.device);
    if (h->stream) cudaStreamSynchronize(h->stream);
    for (void* p : h->g_opened)
        if (p) cudaIpcCloseMemHandle(p);
    void* dev_ptrs[] = {h->kc, h->vc, h->freq, h->qg, h->kg, h->part, h->gpart, h->counters, h->d_stage, h->qf, h->qb,
                        h->d_wm, h->gbuf, h->d_peer_ll, h->d_gstate};
    for (void* p : dev_ptrs)
        if (p) cudaFree(p);
    for (auto* v : {&h->kb, &h->vb})
        for (__nv_bfloat16* p : *v)
            if (p) cudaFree(p);
    if (h->h_err) cudaFreeHost(h->h_err);
    if (h->h_stage) cudaFreeHost(h->h_stage);
    if (h->stream) cudaStreamDestroy(h->stream);
    delete h;
    return LIGGUF_ATTN_OK;
}

int ligguf_cuda_attn_init(const ligguf_attn_cfg* cfg, ligguf_attn** out) {
    if (!cfg || !out) return fail(LIGGUF_ATTN_EINVAL, "null cfg or out");
    *out = nullptr;
    ligguf_attn_cfg c = *cfg;
    if (c.n_layers < 1 || c.n_heads < 1 || c.n_kv_heads < 1 || c.n_context < 1)
        return fail(LIGGUF_ATTN_EINVAL, "n_layers, n_heads, n_kv_heads and n_context must be positive");
    if (c.n_heads % c.n_kv_heads)
        return fail(LIGGUF_ATTN_EINVAL, "n_heads %d is not a multiple of n_kv_heads %d", c.n_heads, c.n_kv_heads);
    if (c.head_dim != 64 && c.head_dim != 128)
        return fail(LIGGUF_ATTN_EUNSUPPORTED, "head_dim %d (supported: 64, 128)", c.head_dim);
    if (c.kv_type < LIGGUF_KV_F32 || c.kv_type > LIGGUF_KV_BF16) return fail(LIGGUF_ATTN_EINVAL, "kv_type %d", c.kv_type);
    if (c.scale_mode != LIGGUF_SCALE_MUL && c.scale_mode != LIGGUF_SCALE_DIV)
        return fail(LIGGUF_ATTN_EINVAL, "scale_mode %d", c.scale_mode);
    if (c.kv_headn == 0) {
        if (c.kv_head0 != 0) return fail(LIGGUF_ATTN_EINVAL, "kv_head0 without kv_headn");
        c.kv_headn = c.n_kv_heads;
    }
    if (c.kv_head0 < 0 || c.kv_headn < 1 || c.kv_head0 + c.kv_headn > c.n_kv_heads)
        return fail(LIGGUF_ATTN_EINVAL, "shard [%d, %d) outside the %d KV heads", c.kv_head0, c.kv_head0 + c.kv_headn,
                    c.n_kv_heads);
    const int nrep = c.n_heads / c.n_kv_heads;
    if (nrep != 1 && nrep != 2 && nrep != 4 && nrep != 8)
        return fail(LIGGUF_ATTN_EUNSUPPORTED, "n_heads/n_kv_heads = %d (supported: 1, 2, 4, 8)", nrep);
    if (c.rope_dim < 0) return fail(LIGGUF_ATTN_EINVAL, "rope_dim %d", c.rope_dim);
    if (static_cast<long long>(c.n_layers) * c.n_context > (1ll << 31) - 1)
        return fail(LIGGUF_ATTN_EINVAL, "n_layers * n_context exceeds 2^31");
    int ndev = 0;
    LG_CUDA(cudaGetDeviceCount(&ndev));
    if (c.device < 0 || c.device >= ndev) return fail(LIGGUF_ATTN_EINVAL, "device %d of %d", c.device, ndev);

    DeviceGuard dg(c.device);
    ligguf_attn* h = new ligguf_attn();
    h->cfg = c;
    h->cfg.rope_freq = nullptr;
    h->nrep = nrep;
    h->q_headn = c.kv_headn * nrep;
    h->kv_dim = c.kv_headn * c.head_dim;
    h->kv_dim_full = c.n_kv_heads * c.head_dim;
    int rd = c.rope_dim > c.head_dim ? c.head_dim : c.rope_dim;  // fast/lil_math.cpp:904-906
    if (rd & 1) rd--;
    h->rope_pairs = rd / 2;
    h->es = kv_elem_size(c.kv_type);
    h->layer_elems = size_t(c.n_context) * h->kv_dim;
    h->norm_set.assign(c.n_layers, 0);
    int rc = LIGGUF_ATTN_OK;
    auto bail = [&](int code) {
        ligguf_cuda_attn_free(h);
        return code;
    };
    if (cudaDeviceGetAttribute(&h->num_sms, cudaDevAttrMultiProcessorCount, c.device) != cudaSuccess)
        return bail(fail(LIGGUF_ATTN_ECUDA, "cudaDeviceGetAttribute failed"));
    if (cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess)
        return bail(fail(LIGGUF_ATTN_ECUDA, "cudaStreamCreate failed"));
    const size_t cache_bytes = size_t(c.n_layers) * h->layer_elems * h->es;
    if (cudaMalloc(&h->kc, cache_bytes) != cudaSuccess || cudaMalloc(&h->vc, cache_bytes) != cudaSuccess)
        return bail(fail(LIGGUF_ATTN_ENOMEM, "KV cache of 2 x %zu bytes does not fit", cache_bytes));
    if (cudaMemset(h->kc, 0, cache_bytes) != cudaSuccess || cudaMemset(h->vc, 0, cache_bytes) != cudaSuccess)
        return bail(fail(LIGGUF_ATTN_ECUDA, "cudaMemset of the cache failed"));
    // RoPE table: the caller's, else powf(base, -2i/rope_dim) as fast/common.cpp:38-39.
    const int nfreq = std::max(1, c.rope_dim / 2);
    std::vector<float> freq(nfreq, 0.f);
    for (int i = 0; i < c.rope_dim / 2; i++)
        freq[i] = cfg->rope_freq ? cfg->rope_freq[i]
                                 : powf(c.rope_base, -2.0f * static_cast<float>(i) / static_cast<float>(c.rope_dim));
    const size_t pd = size_t(c.n_layers) * c.head_dim;
    const size_t part_floats = size_t(c.kv_headn) * lg::kDecodeMaxSplit * lg::decode_part_stride(nrep, c.head_dim);
    const size_t gpart_floats = size_t(c.kv_headn) * lg::kDecodeMaxGroups * lg::decode_part_stride(nrep, c.head_dim);
    const size_t n_counters = size_t(c.kv_headn) * (2 + lg::kDecodeMaxGroups);
    if (cudaMalloc(&h->freq, nfreq * 4) != cudaSuccess || cudaMalloc(&h->qg, pd * 4) != cudaSuccess ||
        cudaMalloc(&h->kg, pd * 4) != cudaSuccess || cudaMalloc(&h->part, part_floats * 4) != cudaSuccess ||
        cudaMalloc(&h->gpart, gpart_floats * 4) != cudaSuccess ||
        cudaMalloc(&h->counters, n_counters * sizeof(int)) != cudaSuccess ||
        cudaMalloc(&h->d_wm, size_t(c.n_layers) * sizeof(int)) != cudaSuccess)
        return bail(fail(LIGGUF_ATTN_ENOMEM, "handle buffers"));
    h->kb.assign(c.n_layers, nullptr);
    h->vb.assign(c.n_layers, nullptr);
    if (cudaMemcpy(h->freq, freq.data(), nfreq * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemset(h->counters, 0, n_counters * sizeof(int)) != cudaSuccess ||
        cudaMemset(h->d_wm, 0, size_t(c.n_layers) * sizeof(int)) != cudaSuccess)
        return bail(fail(LIGGUF_ATTN_ECUDA, "handle initialisation copies"));
    if (cudaHostAlloc(&h->h_err, 64, cudaHostAllocMapped) != cudaSuccess ||
        cudaHostGetDevicePointer(reinterpret_cast<void**>(&h->d_err), h->h_err, 0) != cudaSuccess)
        return bail(fail(LIGGUF_ATTN_ENOMEM, "mapped error word"));
    *h->h_err = 0;
    const int tp = decode_tile_rows(c.kv_type, c.head_dim);
    if ((rc = make_cache_tmap(&h->tm_k, h->kc, h, tp)) != LIGGUF_ATTN_OK) return bail(rc);
    if ((rc = make_cache_tmap(&h->tm_v, h->vc, h, tp)) != LIGGUF_ATTN_OK) return bail(rc);
    *out = h;
    return LIGGUF_ATTN_OK;
}

int ligguf_cuda_attn_set_qk_norm(ligguf_attn* h, int layer, const float* q_gamma, const float* k_gamma) {
    if (!h || !q_gamma || !k_gamma) return fail(LIGGUF_ATTN_EINVAL, "null argument");
    if (layer < 0 || layer >= h->cfg.n_layers) return fail(LIGGUF_ATTN_EINVAL, "layer %d out of range", layer);
    DeviceGuard dg(h->cfg.device);
    const size_t D = h->cfg.head_dim;
    LG_CUDA(cudaMemcpy(h->qg + layer * D, q_gamma, D * 4, cudaMemcpyHostToDevice));
    LG_CUDA(cudaMemcpy(h->kg + layer * D, k_gamma, D * 4, cudaMemcpyHostToDevice));
    h->norm_set[layer] = 1;
    return LIGGUF_ATTN_OK;
}

int ligguf_cuda_attn_decode_async(ligguf_attn* h, int layer, int pos, const float* d_q, const float* d_k,
                                  const float* d_v, float* d_out, void* stream) {
    if (!h) return fail(LIGGUF_ATTN_EINVAL, "null handle");
    DeviceGuard dg(h->cfg.device);
    return decode_enqueue(h, layer, pos, d_q, d_k, d_v, d_out, static_cast<cudaStream_t>(stream), false);
}

// The device address of pinned (page-locked, mapped) host memory, or null for any other pointer.
static void* mapped_host(const void* p) {
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();  // pageable memory unknown to CUDA: not an error for the caller
        return nullptr;
    }
    return at.type == cudaMemoryTypeHost ? at.devicePointer : nullptr;
}

int ligguf_cuda_attn_decode(ligguf_attn* h, int layer, int pos, const float* q, const float* k, const float* v,
                            float* out) {
    if (!h) return fail(LIGGUF_ATTN_EINVAL, "null handle");
    if (!q || !k || !v || !out) return fail(LIGGUF_ATTN_EINVAL, "null tensor pointer");
    DeviceGuard dg(h->cfg.device);
    const size_t nq = size_t(h->q_headn) * h->cfg.head_dim, nk = h->kv_dim;
    int rc = grow(&h->d_stage, &h->stage_floats, 2 * nq + 2 * nk);
    if (rc) return rc;
    // q, k, v are gathered on the host into one pinned buffer and cross in one copy (every CTA of the
    // kernel reads q, so reading it in place over the host link would fetch it hundreds of times).
    // The output is written once, by the last CTA of each KV head, in place over the host link:
    // into the caller's buffer when it is pinned, else into the pinned buffer and copied from there.
    if (h->h_stage_floats < 2 * nq + 2 * nk) {
        if (h->h_stage) cudaFreeHost(h->h_stage);
        h->h_stage = nullptr;
        h->h_stage_floats = 0;
        if (cudaHostAlloc(reinterpret_cast<void**>(&h->h_stage), (2 * nq + 2 * nk) * 4, cudaHostAllocMapped) !=
            cudaSuccess)
            return fail(LIGGUF_ATTN_ENOMEM, "pinned staging of %zu bytes", (2 * nq + 2 * nk) * 4);
        h->h_stage_floats = 2 * nq + 2 * nk;
        LG_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&h->h_stage_dev), h->h_stage, 0));
    }
    std::memcpy(h->h_stage, q, nq * 4);
    std::memcpy(h->h_stage + nq, k, nk * 4);
    std::memcpy(h->h_stage + nq + nk, v, nk * 4);
    LG_CUDA(cudaMemcpyAsync(h->d_stage, h->h_stage, (nq + 2 * nk) * 4, cudaMemcpyHostToDevice, h->stream));
    const float* dq = h->d_stage;
    const float* dk = h->d_stage + nq;
    const float* dv = h->d_stage + nq + nk;
    float* dout = static_cast<float*>(mapped_host(out));
    const bool out_mapped = dout != nullptr;
    if (!out_mapped) dout = h->h_stage_dev + nq + 2 * nk;
    if ((rc = decode_enqueue(h, layer, pos, dq, dk, dv, dout, h->stream, false))) return rc;
    LG_CUDA(cudaStreamSynchronize(h->stream));
    if (!out_mapped) std::memcpy(out, h->h_stage + nq + 2 * nk, nq * 4);
    return check_err_word(h->h_err, h->counters, (2 + lg::kDecodeMaxGroups) * h->kv_dim / h->cfg.head_dim);
}

int ligguf_cuda_attn_prefill_async(ligguf_attn* h, int layer, int pos0, int n, const float* d_q, const float* d_k,
                                   const float* d_v, float* d_out, int mode, void* stream) {
    if (!h) return fail(LIGGUF_ATTN_EINVAL, "null handle");
    DeviceGuard dg(h->cfg.device);
    return prefill_enqueue(h, layer, pos0, n, d_q, d_k, d_v, d_out, mode, static_cast<cudaStream_t>(stream));
}

int ligguf_cuda_attn_prefill(ligguf_attn* h, int layer, int pos0, int n, const float* q, const float* k,
                             const float* v, float* out, int mode) {
    if (!h) return fail(LIGGUF_ATTN_EINVAL, "null handle");
    if (!q || !k || !v || !out || n < 1) return fail(LIGGUF_ATTN_EINVAL, "null tensor pointer or n < 1");
    DeviceGuard dg(h->cfg.device);
    const size_t nq = size_t(n) * h->q_headn * h->cfg.head_dim, nk = size_t(n) * h->kv_dim;
    int rc = grow(&h->d_stage, &h->stage_floats, 2 * nq + 2 * nk);
    if (rc) return rc;
    float* dq = h->d_stage;
    float* dk = dq + nq;
    float* dv = dk + nk;
    float* dout = dv + nk;
    LG_CUDA(cudaMemcpyAsync(dq, q, nq * 4, cudaMemcpyHostToDevice, h->stream));
    LG_CUDA(cudaMemcpyAsync(dk, k, nk * 4, cudaMemcpyHostToDevice, h->stream));
    LG_CUDA(cudaMemcpyAsync(dv, v, nk * 4, cudaMemcpyHostToDevice, h->stream));
    if ((rc = prefill_enqueue(h, layer, pos0, n, dq, dk, dv, dout, mode, h->stream))) return rc;
    LG_CUDA(cudaMemcpyAsync(out, dout, nq * 4, cudaMemcpyDeviceToHost, h->stream));
    LG_CUDA(cudaStreamSynchronize(h->stream));
    return check_err_word(h->h_err, h->counters, (2 + lg::kDecodeMaxGroups) * h->kv_dim / h->cfg.head_dim);
}

int ligguf_cuda_attn_kv_download(ligguf_attn* h, int layer, int pos0, int n, void* host_k, void* host_v) {
    if (!h || !host_k || !host_v) return fail(LIGGUF_ATTN_EINVAL, "null argument");
    if (layer < 0 || layer >= h->cfg.n_layers || pos0 < 0 || n < 0 || pos0 + n > h->cfg.n_context)
        return fail(LIGGUF_ATTN_EINVAL, "layer %d rows [%d, %d) out of range", layer, pos0, pos0 + n);
    DeviceGuard dg(h->cfg.device);
    const size_t off = (size_t(layer) * h->layer_elems + size_t(pos0) * h->kv_dim) * h->es;
    const size_t bytes = size_t(n) * h->kv_dim * h->es;
    LG_CUDA(cudaStreamSynchronize(h->stream));
    LG_CUDA(cudaMemcpy(host_k, static_cast<char*>(h->kc) + off, bytes, cudaMemcpyDeviceToHost));
    LG_CUDA(cudaMemcpy(host_v, static_cast<char*>(h->vc) + off, bytes, cudaMemcpyDeviceToHost));
    return LIGGUF_ATTN_OK;
}

int ligguf_cuda_attn_kv_upload(ligguf_attn* h, int layer, int pos0, int n, const void* host_k, const void* host_v) {
    if (!h || !host_k || !host_v) return fail(LIGGUF_ATTN_EINVAL, "null argument");
    if (layer < 0 || layer >= h->cfg.n_layers || pos0 < 0 || n < 0 || pos0 + n > h->cfg.n_context)
        return fail(LIGGUF_ATTN_EINVAL, "layer %d rows [%d, %d) out of range", layer, pos0, pos0 + n);
    DeviceGuard dg(h->cfg.device);
    const size_t off = (size_t(layer) * h->layer_elems + size_t(pos0) * h->kv_dim) * h->es;
    const size_t bytes = size_t(n) * h->kv_dim * h->es;
    LG_CUDA(cudaStreamSynchronize(h->stream));
    note_cache_write(h, layer, 1, pos0);
    if (int rc = lower_shadow_marks(h, layer, 1, pos0)) return rc;
    LG_CUDA(cudaMemcpy(static_cast<char*>(h->kc) + off, host_k, bytes, cudaMemcpyHostToDevice));
    LG_CUDA(cudaMemcpy(static_cast<char*>(h->vc) + off, host_v, bytes, cudaMemcpyHostToDevice));
    return LIGGUF_ATTN_OK;
}

// ---------------------------------------------------------------------------- FAST state file
// The engine's `model_file` header (fast/common.h:26-31): packed, 24 bytes.
#pragma pack(push, 1)
struct FastStateHeader {
    int pos;
    int n_context;
    uint64_t kv_size;      // cache elements per tensor over all layers: n_layers * pos * kv_dim
    uint64_t logits_size;  // fp32 logits after the cache
};
#pragma pack(pop)
static_assert(sizeof(FastStateHeader) == 24, "model_file header is 24 packed bytes");

static int state_handle_check(const ligguf_attn* h, const char* path) {
    if (!h || !path) return fail(LIGGUF_ATTN_EINVAL, "null handle or path");
    if (h->cfg.kv_type != LIGGUF_KV_F16)
        return fail(LIGGUF_ATTN_EUNSUPPORTED, "the engine state file holds fp16 cache rows: needs kv_type F16");
    if (h->kv_dim != h->kv_dim_full)
        return fail(LIGGUF_ATTN_EUNSUPPORTED, "the engine state file holds every KV head: not a shard's handle");
    return LIGGUF_ATTN_OK;
}

int ligguf_cuda_attn_state_save(ligguf_attn* h, const char* path, int pos, const float* logits, uint64_t n_logits) {
    int rc = state_handle_check(h, path);
    if (rc) return rc;
    if (!logits || n_logits == 0 || pos < 1 || pos > h->cfg.n_context)  // fast/ligguf_fast_qk.cpp:268-271
        return fail(LIGGUF_ATTN_EINVAL, "empty state (pos %d, %llu logits): nothing to save", pos,
                    static_cast<unsigned long long>(n_logits));
    DeviceGuard dg(h->cfg.device);
    LG_CUDA(cudaStreamSynchronize(h->stream));
    FILE* f = fopen(path, "wb");
    if (!f) return fail(LIGGUF_ATTN_EINVAL, "cannot create %s", path);
    FastStateHeader hdr{};
    hdr.kv_size = uint64_t(h->cfg.n_layers) * uint64_t(pos) * uint64_t(h->kv_dim);
    hdr.logits_size = n_logits;
    hdr.n_context = h->cfg.n_context;
    hdr.pos = pos;
    bool ok = fwrite(&hdr, sizeof(hdr), 1, f) == 1;
    const size_t bytes = size_t(pos) * h->kv_dim * sizeof(__half);  // one layer's rows [0, pos)
    std::vector<uint8_t> buf(bytes);
    for (int t = 0; t < 2 && ok; ++t) {  // K of every layer, then V (fast/ligguf_fast_qk.cpp:286-293)
        const char* base = static_cast<const char*>(t ? h->vc : h->kc);
        for (int l = 0; l < h->cfg.n_layers && ok; ++l) {
            if (cudaMemcpy(buf.data(), base + size_t(l) * h->layer_elems * h->es, bytes, cudaMemcpyDeviceToHost) !=
                cudaSuccess) {
                (void)cudaGetLastError();
                fclose(f);
                return fail(LIGGUF_ATTN_ECUDA, "cache download for the state file failed");
            }
            ok = fwrite(buf.data(), bytes, 1, f) == 1;
        }
    }
    ok = ok && fwrite(logits, n_logits * sizeof(float), 1, f) == 1;
    ok = (fclose(f) == 0) && ok;
    if (!ok) return fail(LIGGUF_ATTN_EINVAL, "writing %s failed", path);
    return LIGGUF_ATTN_OK;
}

int ligguf_cuda_attn_state_load(ligguf_attn* h, const char* path, int* pos_out, int* n_context_out, float* logits,
                                uint64_t n_logits) {
    int rc = state_handle_check(h, path);
    if (rc) return rc;
    if (!logits || n_logits == 0) return fail(LIGGUF_ATTN_EINVAL, "no logits buffer");
    FILE* f = fopen(path, "rb");
    if (!f) return fail(LIGGUF_ATTN_EINVAL, "cannot read %s", path);
    auto bad = [&](const char* why) {
        fclose(f);
        return fail(LIGGUF_ATTN_EINVAL, "%s: %s", path, why);
    };
    FastStateHeader hdr{};
    if (fread(&hdr, sizeof(hdr), 1, f) != 1) return bad("no header");
    // The reference's checks (fast/ligguf_fast_qk.cpp:228-233,251), then this handle's room.
    if (!hdr.kv_size || !hdr.logits_size || !hdr.pos) return bad("empty state");
    if (hdr.pos < 0 || hdr.pos > h->cfg.n_context) return bad("pos beyond this handle's n_context");
    const uint64_t lsz = uint64_t(hdr.pos) * uint64_t(h->kv_dim);
    if (hdr.kv_size != uint64_t(h->cfg.n_layers) * lsz) return bad("cache size does not match this model");
    if (hdr.logits_size != n_logits) return bad("logits size does not match");
    // The whole file is checked before anything is touched: a short file changes nothing.
    const uint64_t want = sizeof(hdr) + 2 * hdr.kv_size * sizeof(__half) + hdr.logits_size * sizeof(float);
    if (fseek(f, 0, SEEK_END) != 0) return bad("cannot seek");
    const long have = ftell(f);
    if (have < 0 || uint64_t(have) != want) return bad("file size does not match its header");
    if (fseek(f, long(sizeof(hdr)), SEEK_SET) != 0) return bad("cannot seek");
    DeviceGuard dg(h->cfg.device);
    LG_CUDA(cudaStreamSynchronize(h->stream));
    const size_t bytes = size_t(lsz) * sizeof(__half);
    std::vector<uint8_t> buf(bytes);
    for (int t = 0; t < 2; ++t) {  // fast/ligguf_fast_qk.cpp:238-248
        char* base = static_cast<char*>(t ? h->vc : h->kc);
        for (int l = 0; l < h->cfg.n_layers; ++l) {
            if (fread(buf.data(), bytes, 1, f) != 1) return bad("short read of the cache");
            if (cudaMemcpy(base + size_t(l) * h->layer_elems * h->es, buf.data(), bytes, cudaMemcpyHostToDevice) !=
                cudaSuccess) {
                (void)cudaGetLastError();
                fclose(f);
                return fail(LIGGUF_ATTN_ECUDA, "cache upload from the state file failed");
            }
        }
    }
    std::vector<float> lg(n_logits);
    if (fread(lg.data(), n_logits * sizeof(float), 1, f) != 1) return bad("short read of the logits");
    fclose(f);
    note_cache_write(h, 0, h->cfg.n_layers, 0);
    if (int rc = lower_shadow_marks(h, 0, h->cfg.n_layers, 0)) return rc;
    std::memcpy(logits, lg.data(), n_logits * sizeof(float));
    if (pos_out) *pos_out = hdr.pos;
    if (n_context_out) *n_context_out = hdr.n_context;
    return LIGGUF_ATTN_OK;
}

int ligguf_cuda_attn_kv_synth(ligguf_attn* h, int layer0, int n_layers, int pos0, int n, uint64_t seed,
                              float scale) {
    if (!h) return fail(LIGGUF_ATTN_EINVAL, "null handle");
    if (layer0 < 0 || n_layers < 0 || layer0 + n_layers > h->cfg.n_layers || pos0 < 0 || n < 0 ||
        pos0 + n > h->cfg.n_context)
        return fail(LIGGUF_ATTN_EINVAL, "synthetic fill range out of bounds");
    DeviceGuard dg(h->cfg.device);
    const float mul = synth_mul(scale);
    const int kv_off = h->cfg.kv_head0 * h->cfg.head_dim;
    note_cache_write(h, layer0, n_layers, pos0);
    if (int rc = lower_shadow_marks(h, layer0, n_layers, pos0)) return rc;
    const size_t total = size_t(n) * h->kv_dim;
    const int blocks = std::min(8 * h->num_sms, std::max(1, ceil_div(total, 256)));
    for (int l = layer0; l < layer0 + n_layers && n > 0; ++l) {
        for (int tensor = LIGGUF_SYNTH_K; tensor <= LIGGUF_SYNTH_V; ++tensor) {
            void* base = static_cast<char*>(tensor == LIGGUF_SYNTH_K ? h->kc : h->vc) + size_t(l) * h->layer_elems * h->es;
            const uint64_t sb = lg::synth_base(seed, (uint64_t(tensor) << 32) | uint32_t(l));
            switch (h->cfg.kv_type) {
                case LIGGUF_KV_F32:
                    kv_synth_kernel<float><<<blocks, 256, 0, h->stream>>>(static_cast<float*>(base), h->kv_dim,
                                                                          h->kv_dim_full, kv_off, pos0, n, sb, mul);
                    break;
                case LIGGUF_KV_F16:
                    kv_synth_kernel<__half><<<blocks, 256, 0, h->stream>>>(static_cast<__half*>(base), h->kv_dim,
                                                                           h->kv_dim_full, kv_off, pos0, n, sb, mul);
                    break;
                default:
                    kv_synth_kernel<__nv_bfloat16><<<blocks, 256, 0, h->stream>>>(
                        static_cast<__nv_bfloat16*>(base), h->kv_dim, h->kv_dim_full, kv_off, pos0, n, sb, mul);
                    break;
            }
            LG_CUDA(cudaGetLastError());
        }
    }
    LG_CUDA(cudaStreamSynchronize(h->stream));
    return LIGGUF_ATTN_OK;
}

int ligguf_cuda_attn_sync(ligguf_attn* h) {
    if (!h) return fail(LIGGUF_ATTN_EINVAL, "null handle");
    DeviceGuard dg(h->cfg.device);
    LG_CUDA(cudaStreamSynchronize(h->stream));
    LG_CUDA(cudaDeviceSynchronize());
    return check_err_word(h->h_err, h->counters, (2 + lg::kDecodeMaxGroups) * h->kv_dim / h->cfg.head_dim);
}

// ---------------------------------------------------------------------------- SARA gather
int ligguf_cuda_attn_gather_ipc_handle(ligguf_attn* h, void* handle_out, size_t handle_size) {
    if (!h || !handle_out) return fail(LIGGUF_ATTN_EINVAL, "null argument");
    if (handle_size < sizeof(cudaIpcMemHandle_t))
        return fail(LIGGUF_ATTN_EINVAL, "handle buffer of %zu bytes (need %zu)", handle_size, sizeof(cudaIpcMemHandle_t));
    DeviceGuard dg(h->cfg.device);
    if (!h->gbuf) {
        h->gbuf_bytes = 2 * lg::gather_slot_words(h->cfg.n_heads, h->cfg.head_dim) * sizeof(unsigned long long);
        if (cudaMalloc(reinterpret_cast<void**>(&h->gbuf), h->gbuf_bytes) != cudaSuccess)
            return fail(LIGGUF_ATTN_ENOMEM, "gather buffer");
        LG_CUDA(cudaMemset(h->gbuf, 0, h->gbuf_bytes));
    }
    cudaIpcMemHandle_t hd;
    LG_CUDA(cudaIpcGetMemHandle(&hd, h->gbuf));
    memcpy(handle_out, &hd, sizeof(hd));
    return LIGGUF_ATTN_OK;
}

int ligguf_cuda_attn_gather_open(ligguf_attn* h, int nranks, int rank, const void* handles, size_t handle_size) {
    if (!h || !handles) return fail(LIGGUF_ATTN_EINVAL, "null argument");
    if (handle_size < sizeof(cudaIpcMemHandle_t)) return fail(LIGGUF_ATTN_EINVAL, "handle stride %zu", handle_size);
    if (nranks < 1 || rank < 0 || rank >= nranks) return fail(LIGGUF_ATTN_EINVAL, "rank %d of %d", rank, nranks);
    if (!h->gbuf) return fail(LIGGUF_ATTN_ESTATE, "call ligguf_cuda_attn_gather_ipc_handle first");
    if (h->g_nranks) return fail(LIGGUF_ATTN_ESTATE, "gather already open");
    DeviceGuard dg(h->cfg.device);
    const size_t slot_words = lg::gather_slot_words(h->cfg.n_heads, h->cfg.head_dim);
    std::vector<unsigned long long*> slots(2 * nranks);
    h->g_opened.assign(nranks, nullptr);
    for (int r = 0; r < nranks; ++r) {
        unsigned long long* base;
        if (r == rank) {
            base = h->gbuf;
        } else {
            cudaIpcMemHandle_t hd;
            memcpy(&hd, static_cast<const char*>(handles) + size_t(r) * handle_size, sizeof(hd));
            void* p = nullptr;
            LG_CUDA(cudaIpcOpenMemHandle(&p, hd, cudaIpcMemLazyEnablePeerAccess));
            h->g_opened[r] = p;
            base = static_cast<unsigned long long*>(p);
        }
        for (int slot = 0; slot < 2; ++slot) slots[slot * nranks + r] = base + slot * slot_words;
    }
    LG_CUDA(cudaMalloc(reinterpret_cast<void**>(&h->d_peer_ll), slots.size() * sizeof(unsigned long long*)));
    LG_CUDA(cudaMemcpy(h->d_peer_ll, slots.data(), slots.size() * sizeof(unsigned long long*), cudaMemcpyHostToDevice));
    LG_CUDA(cudaMalloc(reinterpret_cast<void**>(&h->d_gstate), 2 * sizeof(int)));
    LG_CUDA(cudaMemset(h->d_gstate, 0, 2 * sizeof(int)));
    h->g_nranks = nranks;
    h->g_rank = rank;
    h->g_pending = false;
    return LIGGUF_ATTN_OK;
}

int ligguf_cuda_attn_decode_gather_async(ligguf_attn* h, int layer, int pos, const float* d_q, const float* d_k,
                                         const float* d_v, void* stream) {
    if (!h) return fail(LIGGUF_ATTN_EINVAL, "null handle");
    if (!h->g_nranks) return fail(LIGGUF_ATTN_ESTATE, "gather not open");
    if (h->g_pending) return fail(LIGGUF_ATTN_ESTATE, "the previous gathered decode has no gather wait yet");
    DeviceGuard dg(h->cfg.device);
    const int rc = decode_enqueue(h, layer, pos, d_q, d_k, d_v, nullptr, static_cast<cudaStream_t>(stream), true);
    if (!rc) h->g_pending = true;
    return rc;
}

int ligguf_cuda_attn_gather_wait_async(ligguf_attn* h, int layer, float* d_out, void* stream) {
    if (!h || !d_out) return fail(LIGGUF_ATTN_EINVAL, "null argument");
    if (!h->g_nranks || !h->g_pending) return fail(LIGGUF_ATTN_ESTATE, "no gathered decode in flight");
    if (layer < 0 || layer >= h->cfg.n_layers) return fail(LIGGUF_ATTN_EINVAL, "layer %d out of range", layer);
    DeviceGuard dg(h->cfg.device);
    const int vec = h->cfg.n_heads * h->cfg.head_dim;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(ceil_div(vec, 256), 1, 1);
    lc.blockDim = dim3(256, 1, 1);
    lc.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    LG_CUDA(cudaLaunchKernelEx(&lc, gather_wait_kernel, static_cast<const unsigned long long*>(h->gbuf), h->d_gstate,
                               d_out, h->cfg.n_heads, h->cfg.head_dim, h->d_err));
    LG_CUDA(cudaGetLastError());
    h->g_pending = false;
    return LIGGUF_ATTN_OK;
}

// ---------------------------------------------------------------------------- BERT
int ligguf_cuda_bert_free(ligguf_bert_attn* b) {
    if (!b) return LIGGUF_ATTN_OK;
    DeviceGuard dg(b->device);
    if (b->stream) cudaStreamSynchronize(b->stream);
    if (b->d_lens) cudaFree(b->d_lens);
    if (b->d_buf) cudaFree(b->d_buf);
    if (b->bf) cudaFree(b->bf);
    if (b->d_order) cudaFree(b->d_order);
    if (b->h_err) cudaFreeHost(b->h_err);
    if (b->stream) cudaStreamDestroy(b->stream);
    delete b;
    return LIGGUF_ATTN_OK;
}

int ligguf_cuda_bert_init(int n_heads, int head_dim, int max_batch, int max_len, int device, ligguf_bert_attn** out) {
    if (!out) return fail(LIGGUF_ATTN_EINVAL, "null out");
    *out = nullptr;
    if (n_heads < 1 || max_batch < 1 || max_len < 1) return fail(LIGGUF_ATTN_EINVAL, "non-positive size");
    if (head_dim != 64 && head_dim != 128) return fail(LIGGUF_ATTN_EUNSUPPORTED, "head_dim %d", head_dim);
    int ndev = 0;
    LG_CUDA(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev) return fail(LIGGUF_ATTN_EINVAL, "device %d of %d", device, ndev);
    DeviceGuard dg(device);
    ligguf_bert_attn* b = new ligguf_bert_attn();
    b->n_heads = n_heads;
    b->head_dim = head_dim;
    b->max_batch = max_batch;
    b->max_len = max_len;
    b->device = device;
    const size_t elems = size_t(max_batch) * max_len * n_heads * head_dim;
    if (cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&b->d_lens, max_batch * sizeof(int)) != cudaSuccess ||
        cudaHostAlloc(&b->h_err, 64, cudaHostAllocMapped) != cudaSuccess ||
        cudaHostGetDevicePointer(reinterpret_cast<void**>(&b->d_err), b->h_err, 0) != cudaSuccess) {
        ligguf_cuda_bert_free(b);
        return fail(LIGGUF_ATTN_ENOMEM, "BERT handle buffers");
    }
    (void)elems;
    *b->h_err = 0;
    *out = b;
    return LIGGUF_ATTN_OK;
}

// q, k, v (fp32, [batch][max_len][E]) to the bf16 operands of the tensor-core path, valid rows only
// (one pass; padded v rows zeroed).  E is n_heads * head_dim, a multiple of 64.  The same launch
// writes the tensor-core kernel's work order into `order` (bert_order_ints(...) ints) when it is
// not null.
static cudaError_t bert_convert(const float* q, const float* k, const float* v, const int* lens, int batch,
                               int max_len, int n_heads, int head_dim, __nv_bfloat16* bq, __nv_bfloat16* bk,
                               __nv_bfloat16* bv, int* order, cudaStream_t st) {
    const dim3 grid(ceil_div(max_len, lg::kBertConvRows) + (order ? 1 : 0), batch);
    lg::bert_to_bf16_kernel<<<grid, 256, 0, st>>>(q, k, v, lens, max_len, n_heads * head_dim, bq, bk, bv, n_heads,
                                                  order);
    return cudaGetLastError();
}

// Length of the work order of a BERT batch (one int per tensor-core work item), or 0 when the
// lengths could reach more key tiles than the order's counting sort has bins for (then the kernel
// walks its items in their natural order).
static size_t bert_order_ints(int n_heads, int batch, int max_len) {
    if (ceil_div(max_len, lg::kTcKeys) >= lg::kOrderBins) return 0;
    return size_t(n_heads) * ceil_div(max_len, lg::kTcRows) * batch;
}

int ligguf_cuda_bert_attn_async(ligguf_bert_attn* b, int batch, int max_len, const int* d_lens, const float* d_q,
                                const float* d_k, const float* d_v, float* d_out, int mode, void* stream) {
    if (!b || !d_lens || !d_q || !d_k || !d_v || !d_out) return fail(LIGGUF_ATTN_EINVAL, "null argument");
    if (batch < 1 || batch > b->max_batch || max_len < 1 || max_len > b->max_len)
        return fail(LIGGUF_ATTN_EINVAL, "batch %d / max_len %d beyond the handle's %d / %d", batch, max_len,
                    b->max_batch, b->max_len);
    if (mode != LIGGUF_MODE_SIMT && mode != LIGGUF_MODE_TC) return fail(LIGGUF_ATTN_EINVAL, "mode %d", mode);
    DeviceGuard dg(b->device);
    const int D = b->head_dim, E = b->n_heads * D;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (mode == LIGGUF_MODE_SIMT) {
        lg::FlashArgs f = {};
        f.q = d_q;
        f.q_row = E;
        f.q_batch = static_cast<long long>(max_len) * E;
        f.k = d_k;
        f.v = d_v;
        f.kv_row = E;
        f.kv_batch = static_cast<long long>(max_len) * E;
        f.out = d_out;
        f.o_row = E;
        f.o_batch = static_cast<long long>(max_len) * E;
        f.lens = d_lens;
        f.n_q = max_len;
        f.kv_len = max_len;
        f.causal = 0;
        f.q_pos0 = 0;
        f.nrep = 1;
        f.scale_div = 0;
        f.scale = 1.0f / sqrtf(static_cast<float>(D));  // fast/vdb.cpp:133
        return launch_flash_simt<float>(f, D, dim3(ceil_div(max_len, lg::kFlashBQ), b->n_heads, batch), st, b->device);
    }
    const size_t elems = size_t(batch) * max_len * E;
    size_t cap = b->bf ? size_t(b->max_batch) * b->max_len * E * 3 : 0;
    if (!b->bf) {
        cap = size_t(b->max_batch) * b->max_len * E * 3;
        if (cudaMalloc(&b->bf, cap * sizeof(__nv_bfloat16)) != cudaSuccess)
            return fail(LIGGUF_ATTN_ENOMEM, "BERT bf16 operand buffers");
        const size_t oc = bert_order_ints(b->n_heads, b->max_batch, b->max_len);
        if (oc && cudaMalloc(&b->d_order, oc * sizeof(int)) != cudaSuccess)
            return fail(LIGGUF_ATTN_ENOMEM, "BERT work-order buffer");
    }
    // A smaller batch or max_len never needs more order entries than the handle's maxima.
    int* order = bert_order_ints(b->n_heads, batch, max_len) ? b->d_order : nullptr;
    lg::TcArgs t = {};
    t.q = b->bf;
    t.k = b->bf + elems;
    t.v = b->bf + 2 * elems;
    t.order = order;
    LG_CUDA(bert_convert(d_q, d_k, d_v, d_lens, batch, max_len, b->n_heads, D, b->bf, b->bf + elems,
                         b->bf + 2 * elems, order, st));
    t.out = d_out;
    t.q_rows = batch * max_len;
    t.q_heads = b->n_heads;
    t.kv_rows = batch * max_len;
    t.kv_heads = b->n_heads;
    t.batch = batch;
    t.q_seq = max_len;
    t.kv_seq = max_len;
    t.lens = d_lens;
    t.causal = 0;
    t.q_pos0 = 0;
    t.nrep = 1;
    t.scale_log2 = (1.0f / sqrtf(static_cast<float>(D))) * 1.4426950408889634f;
    t.err = b->d_err;
    return launch_flash_tc(t, D, st, b->device);
}

int ligguf_cuda_bert_attn(ligguf_bert_attn* b, int batch, int max_len, const int* lens, const float* q,
                          const float* k, const float* v, float* out, int mode) {
    if (!b || !lens || !q || !k || !v || !out) return fail(LIGGUF_ATTN_EINVAL, "null argument");
    if (batch < 1 || batch > b->max_batch || max_len < 1 || max_len > b->max_len)
        return fail(LIGGUF_ATTN_EINVAL, "batch %d / max_len %d beyond the handle's %d / %d", batch, max_len,
                    b->max_batch, b->max_len);
    for (int i = 0; i < batch; ++i)
        if (lens[i] < 0 || lens[i] > max_len) return fail(LIGGUF_ATTN_EINVAL, "lens[%d] = %d", i, lens[i]);
    DeviceGuard dg(b->device);
    const size_t elems = size_t(batch) * max_len * b->n_heads * b->head_dim;
    if (!b->d_buf) {
        const size_t cap = size_t(b->max_batch) * b->max_len * b->n_heads * b->head_dim * 4;
        if (cudaMalloc(&b->d_buf, cap * sizeof(float)) != cudaSuccess)
            return fail(LIGGUF_ATTN_ENOMEM, "BERT staging buffers");
    }
    float* dq = b->d_buf;
    float* dk = dq + elems;
    float* dv = dk + elems;
    float* dout = dv + elems;
    LG_CUDA(cudaMemcpyAsync(b->d_lens, lens, batch * sizeof(int), cudaMemcpyHostToDevice, b->stream));
    LG_CUDA(cudaMemcpyAsync(dq, q, elems * 4, cudaMemcpyHostToDevice, b->stream));
    LG_CUDA(cudaMemcpyAsync(dk, k, elems * 4, cudaMemcpyHostToDevice, b->stream));
    LG_CUDA(cudaMemcpyAsync(dv, v, elems * 4, cudaMemcpyHostToDevice, b->stream));
    int rc = ligguf_cuda_bert_attn_async(b, batch, max_len, b->d_lens, dq, dk, dv, dout, mode, b->stream);
    if (rc) return rc;
    LG_CUDA(cudaMemcpyAsync(out, dout, elems * 4, cudaMemcpyDeviceToHost, b->stream));
    LG_CUDA(cudaStreamSynchronize(b->stream));
    return check_err_word(b->h_err, nullptr, 0);
}

// ---------------------------------------------------------------------------- BERT, no allocation
int ligguf_cuda_bert_attn_tc_noalloc(int n_heads, int head_dim, int batch, int max_len, const int* d_lens,
                                     const float* d_q, const float* d_k, const float* d_v, float* d_out,
                                     void* stream) {
    if (!d_lens || !d_q || !d_k || !d_v || !d_out) return fail(LIGGUF_ATTN_EINVAL, "null argument");
    if (n_heads < 1 || batch < 1 || max_len < 1) return fail(LIGGUF_ATTN_EINVAL, "non-positive size");
    if (head_dim != 64 && head_dim != 128) return fail(LIGGUF_ATTN_EUNSUPPORTED, "head_dim %d", head_dim);
    const size_t elems = size_t(batch) * max_len * n_heads * head_dim;
    if (elems > size_t(LIGGUF_NOALLOC_MAX_ELEMS))
        return fail(LIGGUF_ATTN_EINVAL,
                    "batch*max_len*n_heads*head_dim = %zu exceeds the no-allocation limit of %d elements per "
                    "tensor (LIGGUF_NOALLOC_MAX_ELEMS); use ligguf_cuda_bert_attn_async",
                    elems, LIGGUF_NOALLOC_MAX_ELEMS);
    int device = 0;
    LG_CUDA(cudaGetDevice(&device));
    unsigned char* base = nullptr;
    int rc = noalloc_scratch(device, &base);
    if (rc) return rc;
    __nv_bfloat16* bq = reinterpret_cast<__nv_bfloat16*>(base);
    __nv_bfloat16* bk = reinterpret_cast<__nv_bfloat16*>(base + kNoallocOperandBytes);
    __nv_bfloat16* bv = reinterpret_cast<__nv_bfloat16*>(base + 2 * kNoallocOperandBytes);
    int* err = reinterpret_cast<int*>(base + 3 * kNoallocOperandBytes);
    const size_t n_order = bert_order_ints(n_heads, batch, max_len);
    int* order = n_order && n_order <= kNoallocOrderInts
                     ? reinterpret_cast<int*>(base + 3 * kNoallocOperandBytes + 256)
                     : nullptr;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    LG_CUDA(cudaMemsetAsync(err, 0, sizeof(int), st));  // the previous call's error word must not leak
    LG_CUDA(bert_convert(d_q, d_k, d_v, d_lens, batch, max_len, n_heads, head_dim, bq, bk, bv, order, st));
    lg::TcArgs t = {};
    t.q = bq;
    t.k = bk;
    t.v = bv;
    t.order = order;
    t.out = d_out;
    t.q_rows = batch * max_len;
    t.q_heads = n_heads;
    t.kv_rows = batch * max_len;
    t.kv_heads = n_heads;
    t.batch = batch;
    t.q_seq = max_len;
    t.kv_seq = max_len;
    t.lens = d_lens;
    t.causal = 0;
    t.q_pos0 = 0;
    t.nrep = 1;
    t.scale_log2 = (1.0f / sqrtf(static_cast<float>(head_dim))) * 1.4426950408889634f;
    t.err = err;
    return launch_flash_tc(t, head_dim, st, device);
}

int ligguf_cuda_bert_attn_tc_noalloc_status(void* stream) {
    int device = 0;
    LG_CUDA(cudaGetDevice(&device));
    unsigned char* base = nullptr;
    int rc = noalloc_scratch(device, &base);
    if (rc) return rc;
    int* err = reinterpret_cast<int*>(base + 3 * kNoallocOperandBytes);
    LG_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
    int code = 0;
    LG_CUDA(cudaMemcpy(&code, err, sizeof(int), cudaMemcpyDeviceToHost));
    if (code) {
        LG_CUDA(cudaMemset(err, 0, sizeof(int)));
        return fail(LIGGUF_ATTN_ETIMEDOUT,
                    "a bounded wait in the no-allocation BERT kernel gave up (kernel error code %d); its output "
                    "was not written",
                    code);
    }
    return LIGGUF_ATTN_OK;
}

// ---------------------------------------------------------------------------- synth
int ligguf_cuda_synth_fill(void* d_dst, int dtype, size_t n, uint64_t seed, uint64_t stream_id, uint64_t idx0,
                           float scale, float add, void* stream) {
    if (!d_dst && n) return fail(LIGGUF_ATTN_EINVAL, "null destination");
    if (dtype < LIGGUF_KV_F32 || dtype > LIGGUF_KV_BF16) return fail(LIGGUF_ATTN_EINVAL, "dtype %d", dtype);
    if (!n) return LIGGUF_ATTN_OK;
    const uint64_t base = lg::synth_base(seed, stream_id);
    const float mul = synth_mul(scale);
    const int blocks = static_cast<int>(std::min<size_t>(4096, (n + 255) / 256));
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (dtype) {
        case LIGGUF_KV_F32:
            synth_fill_kernel<float><<<blocks, 256, 0, st>>>(static_cast<float*>(d_dst), n, base, idx0, mul, add);
            break;
        case LIGGUF_KV_F16:
            synth_fill_kernel<__half><<<blocks, 256, 0, st>>>(static_cast<__half*>(d_dst), n, base, idx0, mul, add);
            break;
        default:
            synth_fill_kernel<__nv_bfloat16>
                <<<blocks, 256, 0, st>>>(static_cast<__nv_bfloat16*>(d_dst), n, base, idx0, mul, add);
            break;
    }
    LG_CUDA(cudaGetLastError());
    return LIGGUF_ATTN_OK;
}

}  // extern "C"
