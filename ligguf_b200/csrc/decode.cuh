// decode.cuh - single-token decode attention over the HBM-resident KV cache (split-KV
// flash-decoding), one launch per layer.
//
// Replaces fast/ligguf_fast_qk.cpp:42-105 (FAST, fp16 cache) and cpp/ligguf.cpp:674-718 /
// cpp/ligguf_distrib.cpp:724-747 (fp32 cache):
//   q, k <- RMSNorm per head (Qwen3, fast/ligguf_fast_qk.cpp:42-51; fast/lil_math.cpp:931-937)
//   q, k <- RoPE on adjacent pairs at `pos` (fast/lil_math.cpp:901-920)
//   cache[pos] <- k, v (fast/ligguf_fast_qk.cpp:57-62)
//   for each q head h (kv head h/nrep): s_t = q.k_t * scale, softmax over t in [0,pos],
//   out_h = sum_t p_t v_t, with t == pos taken from the fp32 k, v (:77-78, :98-99).
//
// Grid (n_split, kv_headn), one resident wave.  CTA (split, g) works on KV head g: it starts on a
// static chunk of 16 KB tiles of cached positions [0, pos) and then takes further chunks of the
// head from an atomic counter (so CTAs that stream faster take more tiles; one static wave left SMs
// idle for a fifth of the kernel at 32K).  When each CTA has only a few tiles (short contexts, or
// one KV head per GPU), the static chunks cover everything instead: no grabs, and the first
// kDecodeEarlyTiles tiles of a chunk are requested before the previous kernel in the stream has
// finished.  A CTA computes all nrep q heads of the group, so each K/V byte is
// read from HBM once.  Warp 8 is the producer: one lane grabs chunks and streams their K and V tiles
// with TMA into a 3-stage shared-memory ring, publishing each stage's tile index in shared memory.  Warps 0..7 consume: scores (each lane dots 16 B of a row with
// the nrep q vectors, a transposed butterfly reduces nrep*4 dot products with one shuffle per
// result), an online softmax per tile, P.V accumulation in registers.  The last CTA of a KV head
// (atomic ticket) merges the splits' (max, sum, o) partials and writes the output, so the whole
// layer is one launch.  The CTA holding position pos-1 also folds in the current token.  A gathered
// (multi-GPU) decode with many splits stops after the first merge level: each group's merger stores
// the group's (max, sum, o) into every rank's gather slot, and the gather wait merges the groups.
//
// Every wait is bounded (kWaitLimitNs): a wait that gives up raises a shared abort flag, writes the
// error word and lets the kernel finish without writing its output.
#pragma once

#include "common.cuh"

namespace lg {

constexpr int kDecodeConsumerWarps = 8;
constexpr int kDecodeConsumers = kDecodeConsumerWarps * 32;
constexpr int kDecodeThreads = kDecodeConsumers + 32;
constexpr int kDecodeStages = 3;
constexpr int kDecodeTileBytes = 16384;
constexpr int kDecodeMaxSplit = 1024;
constexpr int kDecodeMaxGroups = 32;   // first-level merge groups per KV head (the host bounds n_split)
constexpr int kDecodeStaticMaxTiles = 8;  // up to this many tiles per CTA: static chunks, no grabs
// Tiles a CTA requests before the previous grid completes.  Enough to cover that grid's tail; more
// compete with the tail (its partials, tickets and merge) for memory (4K: 3 tiles 13.5 us per
// layer, 2 tiles 13.0, 1 tile 13.2; one-KV-head 32K shard 16.3 / 15.7 / 15.5; 32K unchanged).
constexpr int kDecodeEarlyTiles = 2;

// One partial (o[NREP][D], m[NREP], l[NREP]) in floats, padded to 16 bytes so that a run of
// partials can be fetched with one bulk copy.
__host__ __device__ constexpr int decode_part_stride(int nrep, int d) { return (nrep * (d + 2) + 3) & ~3; }
// Split partials merged by one CTA: as many as fit the tile ring (the merge copies them there), at
// most 48.
__host__ __device__ constexpr int decode_merge_group(int nrep, int d) {
    return (kDecodeStages * 2 * kDecodeTileBytes) / (decode_part_stride(nrep, d) * 4) < 48
               ? (kDecodeStages * 2 * kDecodeTileBytes) / (decode_part_stride(nrep, d) * 4)
               : 48;
}

// Multi-GPU gather words.  With up to kGatherGroups first-level merge groups per KV head, a gathered
// decode stores each group's (o, m, l) and the gather wait on every rank merges them, instead of a
// second merge level on the shard's GPU.
constexpr int kGatherGroups = 8;
// One gather slot (one per epoch parity), in 64-bit words, for `heads` q heads of `d`:
//   o[kGatherGroups][heads * d]   group results (unnormalised), or the output in group 0
//   m[kGatherGroups][heads], l[kGatherGroups][heads]
//   cnt[heads]                    the number of groups the head's words carry (1: normalised output)
// padded to 32 words, so that both slots start on 256 bytes (the o words take 16-byte stores).
__host__ __device__ constexpr size_t gather_slot_words(int heads, int d) {
    return (size_t(kGatherGroups) * heads * d + 2 * size_t(kGatherGroups) * heads + heads + 31) & ~size_t(31);
}
__host__ __device__ constexpr size_t gather_m_off(int heads, int d) { return size_t(kGatherGroups) * heads * d; }
__host__ __device__ constexpr size_t gather_l_off(int heads, int d) {
    return gather_m_off(heads, d) + size_t(kGatherGroups) * heads;
}
__host__ __device__ constexpr size_t gather_cnt_off(int heads, int d) {
    return gather_l_off(heads, d) + size_t(kGatherGroups) * heads;
}

struct DecodeArgs {
    const float* q;     // [q_headn][D] raw q of this layer
    const float* k;     // [kv_headn][D] raw k
    const float* v;     // [kv_headn][D] raw v
    const float* qg;    // [D] q norm weight (qk_norm) or null
    const float* kg;    // [D]
    const float* freq;  // RoPE inverse frequencies
    void* kc;           // this layer's K cache block [n_context][kv_dim]
    void* vc;
    float* out;         // [q_headn][D]
    float* part;        // [kv_headn][kDecodeMaxSplit][decode_part_stride] split partials
    float* gpart;       // [kv_headn][kDecodeMaxGroups][decode_part_stride] merged group partials
    int* counters;      // [kv_headn] head tickets, then [kv_headn] grab counters, then
                        // [kv_headn][kDecodeMaxGroups] group tickets; zero between launches
    int* err;           // error word (mapped host memory)
    int* shadow_wm;     // the layer's bf16-shadow watermark (tensor-core prefill): lowered to pos
    unsigned long long* const* peer_ll;  // multi-GPU gather (or null): [2][nranks] gather slots of
                                         // gather_slot_words(g_heads, D) words, slot = call epoch & 1
    int nranks;
    int rank;
    int g_heads;        // q heads of the whole model (the gathered vector holds g_heads * D)
    int q_off;          // element offset of this shard's heads in the gathered vector
    int kv_head0;       // global index of this shard's first KV head (gather flag slot)
    const int* epoch;   // gather: the last completed call's epoch (device); this call's is one more
    int pre_rows;       // cache rows [0, pre_rows) of this layer are final before the previous grid ends
    int row0;           // tensor-map row of (this layer, position 0) = layer * n_context
    int pos;
    int n_tiles;        // tiles covering [0, pos)
    int chunk;          // tiles per grab: CTA `split` starts with tiles [split*chunk, +chunk), then takes
                        // further chunks from chunk_ctr[g] (first dynamic chunk = n_split*chunk)
    int dynamic;        // 0: the static chunks cover all tiles (n_split*chunk >= n_tiles), no grabs
    int* chunk_ctr;     // = counters + kv_headn
    int n_split;
    int merge_group;    // splits per first-level merge group (at most decode_merge_group)
    int kv_dim;
    int rope_pairs;
    int qk_norm;
    int scale_div;
    float scale;        // multiplier (FAST) or divisor (cpp/SARA engines)
    float eps;
};

// 2^x on the MUFU (ex2.approx.ftz: relative error about 2^-22; -inf gives +0).
__device__ __forceinline__ float decode_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
constexpr float kLog2e = 1.4426950408889634f;  // log2(e): e^x = 2^(x log2 e)

template <typename KV, int D>
struct DecodeShape {
    static constexpr int kRowBytes = D * static_cast<int>(sizeof(KV));
    static constexpr int kTileRows = kDecodeTileBytes / kRowBytes;
    static constexpr int kLanesPerRow = kRowBytes / 16;
    static constexpr int kRowsPerInstr = 32 / kLanesPerRow;
    static constexpr int kEpl = 16 / static_cast<int>(sizeof(KV));
    static constexpr int kInstr = kTileRows / (kDecodeConsumerWarps * kRowsPerInstr);
    static constexpr int kLog2Lpr = kLanesPerRow == 32 ? 5 : kLanesPerRow == 16 ? 4 : 3;
    static_assert(kRowBytes >= 128 && kRowBytes <= 512, "one head row must be 128..512 bytes");
    static_assert(kInstr == 4, "tile mapping expects 4 row loads per warp per tile");
    static_assert(kDecodeEarlyTiles <= kDecodeStages, "early copies fill at most the ring");
};

template <typename KV, int D, int NREP>
struct DecodeSmem {
    using Sh = DecodeShape<KV, D>;
    static constexpr size_t kStageBytes = 2 * kDecodeTileBytes;  // K tile + V tile
    static constexpr size_t kTilesBytes = kDecodeStages * kStageBytes;
    static constexpr size_t kScoreOff = kTilesBytes;
    static constexpr size_t kScoreBytes = 2 * NREP * Sh::kTileRows * 4;
    static constexpr size_t kQOff = kScoreOff + kScoreBytes;
    static constexpr size_t kOOff = kQOff + NREP * D * 4;
    static constexpr size_t kKnOff = kOOff + NREP * D * 4;
    static constexpr size_t kVnOff = kKnOff + D * 4;
    static constexpr size_t kMiscOff = kVnOff + D * 4;  // corr, m, l [NREP] + 4 ints + stage tile ids
    static constexpr size_t kBarOff = (kMiscOff + 3 * NREP * 4 + 16 + 4 * kDecodeStages + 7) & ~size_t(7);
    static constexpr size_t kTotal = kBarOff + (3 * kDecodeStages + 1) * 8;  // + the merge barrier
    static constexpr int kMergeGroup = decode_merge_group(NREP, D);
    static_assert((kDecodeConsumerWarps * NREP * D + kDecodeConsumerWarps * 2 * NREP) * 4 <= kTilesBytes,
                  "reduction buffer alias");
    static_assert(size_t(kMergeGroup) * decode_part_stride(NREP, D) * 4 <= kTilesBytes, "merge copy fits the ring");
    static_assert(kMergeGroup * NREP <= 2 * NREP * Sh::kTileRows, "merge weights fit the score buffer");
};

// One warp: optional RMSNorm then RoPE of one head (D floats) from global `src` into `dst`.
// Lane owns the adjacent pairs m = lane + 32u, i.e. elements (2m, 2m+1).
template <int D>
__device__ __forceinline__ void norm_rope_head(const float* __restrict__ src,
                                               const float* __restrict__ gamma, int norm,
                                               float eps, const float* __restrict__ freq,
                                               int rope_pairs, int pos, float* dst, int lane) {
    constexpr int kPairs = D / 64;
    float2 x[kPairs];
#pragma unroll
    for (int u = 0; u < kPairs; ++u) x[u] = reinterpret_cast<const float2*>(src)[lane + 32 * u];
    if (norm) {
        float ss = 0.f;
#pragma unroll
        for (int u = 0; u < kPairs; ++u) {
            ss = fmaf(x[u].x, x[u].x, ss);
            ss = fmaf(x[u].y, x[u].y, ss);
        }
        ss = warp_sum(ss);
        const float rs = 1.0f / sqrtf(ss / static_cast<float>(D) + eps);
#pragma unroll
        for (int u = 0; u < kPairs; ++u) {
            const int m = lane + 32 * u;
            x[u].x = (x[u].x * rs) * gamma[2 * m];
            x[u].y = (x[u].y * rs) * gamma[2 * m + 1];
        }
    }
#pragma unroll
    for (int u = 0; u < kPairs; ++u) {
        const int m = lane + 32 * u;
        if (m < rope_pairs) {
            float sn, cs;
            sincosf(static_cast<float>(pos) * freq[m], &sn, &cs);
            const float x0 = x[u].x, x1 = x[u].y;
            x[u].x = x0 * cs - x1 * sn;
            x[u].y = x0 * sn + x1 * cs;
        }
    }
#pragma unroll
    for (int u = 0; u < kPairs; ++u) reinterpret_cast<float2*>(dst)[lane + 32 * u] = x[u];
}

// Same as norm_rope_head with the rotation taken from per-position tables cs/sn[rope_pairs]
// (shared by every head of one token).
template <int D>
__device__ __forceinline__ void norm_rope_regs(float2 (&x)[D / 64], const float* __restrict__ gamma, int norm,
                                               float eps, const float* cs, const float* sn, int rope_pairs,
                                               int lane) {
    constexpr int kPairs = D / 64;
    if (norm) {
        float ss = 0.f;
#pragma unroll
        for (int u = 0; u < kPairs; ++u) {
            ss = fmaf(x[u].x, x[u].x, ss);
            ss = fmaf(x[u].y, x[u].y, ss);
        }
        ss = warp_sum(ss);
        const float rs = 1.0f / sqrtf(ss / static_cast<float>(D) + eps);
#pragma unroll
        for (int u = 0; u < kPairs; ++u) {
            const int m = lane + 32 * u;
            x[u].x = (x[u].x * rs) * gamma[2 * m];
            x[u].y = (x[u].y * rs) * gamma[2 * m + 1];
        }
    }
#pragma unroll
    for (int u = 0; u < kPairs; ++u) {
        const int m = lane + 32 * u;
        if (m < rope_pairs) {
            const float c = cs[m], sn_ = sn[m];
            const float x0 = x[u].x, x1 = x[u].y;
            x[u].x = x0 * c - x1 * sn_;
            x[u].y = x0 * sn_ + x1 * c;
        }
    }
}
// One head (D floats at src): optional RMS norm with gamma, then RoPE from a cos/sin table; lane
// holds pairs m = lane + 32 u (elements 2m, 2m+1).  Result to dst.
template <int D>
__device__ __forceinline__ void norm_rope_head_tab(const float* __restrict__ src,
                                                   const float* __restrict__ gamma, int norm, float eps,
                                                   const float* cs, const float* sn, int rope_pairs,
                                                   float* dst, int lane) {
    constexpr int kPairs = D / 64;
    float2 x[kPairs];
#pragma unroll
    for (int u = 0; u < kPairs; ++u) x[u] = reinterpret_cast<const float2*>(src)[lane + 32 * u];
    norm_rope_regs<D>(x, gamma, norm, eps, cs, sn, rope_pairs, lane);
#pragma unroll
    for (int u = 0; u < kPairs; ++u) reinterpret_cast<float2*>(dst)[lane + 32 * u] = x[u];
}

// Prologue inputs of one head.  The norm weights and the rotation (sin, cos of pos * freq) do not
// depend on the previous kernel, so they are loaded and computed before the kernel waits for it; only
// the head's raw values are loaded after.
template <int D>
struct HeadIn {
    float2 x[D / 64];
    float2 gm[D / 64];
    float cs[D / 64], sn[D / 64];  // rotation of each pair (identity where there is none)
};

template <int D>
__device__ __forceinline__ void head_consts(HeadIn<D>& in, const float* __restrict__ gamma, int norm,
                                            const float* __restrict__ freq, int rope_pairs, int pos, int lane) {
#pragma unroll
    for (int u = 0; u < D / 64; ++u) {
        const int m = lane + 32 * u;
        in.gm[u] = norm ? reinterpret_cast<const float2*>(gamma)[m] : make_float2(1.f, 1.f);
        in.cs[u] = 1.f;
        in.sn[u] = 0.f;
        if (m < rope_pairs) sincosf(static_cast<float>(pos) * freq[m], &in.sn[u], &in.cs[u]);
    }
}

template <int D>
__device__ __forceinline__ void head_load(HeadIn<D>& in, const float* __restrict__ src, int lane) {
#pragma unroll
    for (int u = 0; u < D / 64; ++u) in.x[u] = reinterpret_cast<const float2*>(src)[lane + 32 * u];
}

// The arithmetic of norm_rope_head on prefetched inputs.
template <int D>
__device__ __forceinline__ void head_finish(const HeadIn<D>& in, int norm, float eps, int rope_pairs, float* dst,
                                            int lane) {
    constexpr int kPairs = D / 64;
    float2 x[kPairs];
#pragma unroll
    for (int u = 0; u < kPairs; ++u) x[u] = in.x[u];
    if (norm) {
        float ss = 0.f;
#pragma unroll
        for (int u = 0; u < kPairs; ++u) {
            ss = fmaf(x[u].x, x[u].x, ss);
            ss = fmaf(x[u].y, x[u].y, ss);
        }
        ss = warp_sum(ss);
        const float rs = 1.0f / sqrtf(ss / static_cast<float>(D) + eps);
#pragma unroll
        for (int u = 0; u < kPairs; ++u) {
            x[u].x = (x[u].x * rs) * in.gm[u].x;
            x[u].y = (x[u].y * rs) * in.gm[u].y;
        }
    }
#pragma unroll
    for (int u = 0; u < kPairs; ++u) {
        if (lane + 32 * u < rope_pairs) {
            const float x0 = x[u].x, x1 = x[u].y;
            x[u].x = x0 * in.cs[u] - x1 * in.sn[u];
            x[u].y = x0 * in.sn[u] + x1 * in.cs[u];
        }
    }
#pragma unroll
    for (int u = 0; u < kPairs; ++u) reinterpret_cast<float2*>(dst)[lane + 32 * u] = x[u];
}

// Sums V per-lane values over the 2^S lanes that share the upper lane bits, leaving each lane
// with max(1, V >> S) sums: lane j (low S bits) holds value indices [j*VF, j*VF+VF) when V >= 2^S,
// else index j / (2^S / V).  One shuffle per produced sum instead of S per sum.
template <int V, int S>
__device__ __forceinline__ void transposed_reduce(float (&x)[V], int lane) {
#pragma unroll
    for (int k = 0; k < S; ++k) {
        const int o = 1 << (S - 1 - k);
        const int n = V >> k;
        if (n >= 2) {
            const bool upper = (lane & o) != 0;
#pragma unroll
            for (int t = 0; t < V / 2; ++t) {
                if (t < n / 2) {
                    const float send = upper ? x[t] : x[t + n / 2];
                    const float keep = upper ? x[t + n / 2] : x[t];
                    x[t] = keep + __shfl_xor_sync(0xffffffffu, send, o);
                }
            }
        } else {
            x[0] += __shfl_xor_sync(0xffffffffu, x[0], o);
        }
    }
}

// Ticket of a merge level: after a CTA barrier that orders every thread's partial stores, one
// thread's acquire-release add publishes them at GPU scope (release is cumulative over what the
// barrier ordered before it) and, for the last arrival, makes every other CTA's partials visible.
__device__ __forceinline__ int ticket_acq_rel(int* ctr) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(ctr) : "memory");
    return old;
}

// Merges `count` (o, m, l) partials stored at src[i*PS] (PS = decode_part_stride: o[NREP][D],
// m[NREP], l[NREP]) into o_s (unnormalised sum of o*e^(m-M)), m_s (M, the maximum) and l_s (sum of
// l*e^(m-M)).  The partials were just written by other CTAs: one bulk copy brings them all into
// `buf` (the free tile ring) in a single round trip, and the merge then runs from shared memory;
// `w_s` holds count*NREP weights.  All consumer threads take part.  Returns false (error recorded)
// if the copy did not land in time; the copy is drained before returning either way.
template <int NREP, int D>
__device__ __noinline__ bool merge_partials(const float* src, int count, uint8_t* buf, float* w_s, uint64_t* bar,
                                            uint32_t phase, float* o_s, float* m_s, float* l_s, int tid, int warp,
                                            int lane, uint64_t deadline, volatile int* abort, int* err) {
    constexpr int PS = decode_part_stride(NREP, D);
    const float* pb = reinterpret_cast<const float*>(buf);
    // The ring was last written through the generic proxy (the CTA reduction); order those accesses
    // before the copy engine's writes.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    named_bar_sync(1, kDecodeConsumers);
    if (tid == 0) {
        const uint32_t bytes = uint32_t(count) * PS * 4;
        // The other CTAs' stores were made visible (fence + ticket); order them before the async
        // proxy's reads.
        asm volatile("fence.proxy.async.global;" ::: "memory");
        mbar_arrive_expect_tx(bar, bytes);
        constexpr uint32_t kChunk = 16384;
        for (uint32_t off = 0; off < bytes; off += kChunk) {
            const uint32_t n = bytes - off < kChunk ? bytes - off : kChunk;
            asm volatile(
                "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                    smem_u32(buf + off)),
                "l"(reinterpret_cast<const uint8_t*>(src) + off), "r"(n), "r"(smem_u32(bar))
                : "memory");
        }
    }
    bool ok = mbar_wait_bounded(bar, phase, deadline, abort);
    if (!ok) {
        *abort = 1;
        *reinterpret_cast<volatile int*>(err) = KERR_TIMEOUT_FULL;
        const uint64_t dd = deadline + kWaitLimitNs / 2;  // the copy writes this CTA's memory: drain it
        while (!mbar_try_wait(bar, phase) && globaltimer_ns() < dd) {
        }
    }
    named_bar_sync(1, kDecodeConsumers);
    if (*abort) return false;  // raised by any consumer whose wait failed
    if (warp < NREP) {
        const int h = warp;
        float M = -INFINITY;
        for (int sp = lane; sp < count; sp += 32) M = fmaxf(M, pb[sp * PS + NREP * D + h]);
        M = warp_max(M);
        float L = 0.f;
        for (int sp = lane; sp < count; sp += 32) {
            const float mv = pb[sp * PS + NREP * D + h];
            const float w = mv == -INFINITY ? 0.f : expf(mv - M);
            L = fmaf(pb[sp * PS + NREP * D + NREP + h], w, L);
            w_s[sp * NREP + h] = w;
        }
        L = warp_sum(L);
        if (lane == 0) {
            m_s[h] = M;
            l_s[h] = L;
        }
    }
    named_bar_sync(1, kDecodeConsumers);
    // Weighted sum: all of a thread's columns in one pass over the partials (independent loads and
    // two accumulators per column keep the shared-memory latency overlapped).
    constexpr int CPT = (NREP * D + kDecodeConsumers - 1) / kDecodeConsumers;  // columns per thread
    int hh[CPT];
    float acc[CPT][2];
#pragma unroll
    for (int c = 0; c < CPT; ++c) {
        hh[c] = min(tid + c * kDecodeConsumers, NREP * D - 1) / D;
        acc[c][0] = acc[c][1] = 0.f;
    }
#pragma unroll 4
    for (int sp = 0; sp < count; ++sp) {
        const float* row = pb + sp * PS;
        const float* wr = w_s + sp * NREP;
#pragma unroll
        for (int c = 0; c < CPT; ++c) {
            const int idx = tid + c * kDecodeConsumers;
            if (CPT * kDecodeConsumers == NREP * D || idx < NREP * D)
                acc[c][sp & 1] = fmaf(row[idx], wr[hh[c]], acc[c][sp & 1]);
        }
    }
#pragma unroll
    for (int c = 0; c < CPT; ++c) {
        const int idx = tid + c * kDecodeConsumers;
        if (idx < NREP * D) o_s[idx] = acc[c][0] + acc[c][1];
    }
    named_bar_sync(1, kDecodeConsumers);
    return true;
}

template <typename KV, int D, int NREP>
__global__ void __launch_bounds__(kDecodeThreads, (NREP * DecodeShape<KV, D>::kEpl > 32) ? 1 : 2)
    decode_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                  const DecodeArgs a) {
    using Sh = DecodeShape<KV, D>;
    using Sm = DecodeSmem<KV, D, NREP>;
    constexpr int TP = Sh::kTileRows;
    constexpr int LPR = Sh::kLanesPerRow;
    constexpr int RPI = Sh::kRowsPerInstr;
    constexpr int EPL = Sh::kEpl;
    constexpr int NI = Sh::kInstr;
    constexpr int RB = Sh::kRowBytes;
    constexpr int S = Sh::kLog2Lpr;
    constexpr int NV = NI * NREP;

    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* tiles = smem;
    float* sc = reinterpret_cast<float*>(smem + Sm::kScoreOff);  // [2][NREP][TP]
    float* q_s = reinterpret_cast<float*>(smem + Sm::kQOff);     // [NREP][D]
    float* o_s = reinterpret_cast<float*>(smem + Sm::kOOff);     // [NREP][D]
    float* kn_s = reinterpret_cast<float*>(smem + Sm::kKnOff);   // current token k (normed, roped)
    float* vn_s = reinterpret_cast<float*>(smem + Sm::kVnOff);   // current token v
    float* corr_s = reinterpret_cast<float*>(smem + Sm::kMiscOff);
    float* m_s = corr_s + NREP;
    float* l_s = m_s + NREP;
    volatile int* abort_s = reinterpret_cast<volatile int*>(l_s + NREP);
    volatile int* last_s = abort_s + 1;
    volatile int* stop_s = abort_s + 2;
    volatile int* tile_id_s = abort_s + 4;  // [kDecodeStages]: tile held by each stage, -1 = end
    uint64_t* full_k = reinterpret_cast<uint64_t*>(smem + Sm::kBarOff);
    uint64_t* full_v = full_k + kDecodeStages;
    uint64_t* empty = full_v + kDecodeStages;
    uint64_t* merge_bar = empty + kDecodeStages;  // bulk copy of the partials into the ring

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // x = KV head, y = split: consecutive CTAs alternate heads, so every head's CTAs spread over all
    // SMs and the heads (separate tile pools) see the same bandwidth and finish together.
    const int g = blockIdx.x, split = blockIdx.y;
    const uint64_t deadline = globaltimer_ns() + kWaitLimitNs;
    const int t_end = a.pos;  // cached positions are [0, pos); the current token is folded in last
    const bool owner = split == a.n_split - 1;

    if (tid == 0) {
#pragma unroll
        for (int s = 0; s < kDecodeStages; ++s) {
            mbar_init(&full_k[s], 1);
            mbar_init(&full_v[s], 1);
            mbar_init(&empty[s], kDecodeConsumerWarps);
        }
        mbar_init(merge_bar, 1);
        *abort_s = 0;
        *last_s = 0;
        *stop_s = 0;
        fence_mbar_init();
    }
    // The barriers and flags are initialised before any thread waits on the previous grid, so that
    // the producer can start its early copies at once (a CTA barrier after the consumers' wait
    // would hold the producer until the previous grid completes).
    __syncthreads();
    // Launched as a programmatic dependent of the previous kernel in the stream: everything above
    // touches only this CTA's shared memory; every global read (inputs, the partials and counters
    // this kernel shares with other launches, cache rows) comes after the previous grid has
    // completed - except the producer's first copies of cache rows below a.pre_rows, which no
    // kernel still in flight can be writing (see the producer).  The next kernel may then launch:
    // its CTAs take SM slots as this grid's retire.
    // The producer warp waits later (after its early copies) and never triggers: the dependent grid
    // may launch only once every CTA's consumers have seen the previous grid complete (the gather
    // wait that follows a gathered decode reads the epoch its own predecessor wrote).
    // Consumer warps take the first prologue job (a q head, and k / v of the current token on the
    // owner CTA): its constants before the wait, its raw values right after; the norm and rotation
    // happen after the set-up barrier.
    const int njobs = NREP + (owner ? 2 : 0);
    const bool first_job = warp < kDecodeConsumerWarps && warp < njobs;
    HeadIn<D> pin;
    if (first_job)
        head_consts<D>(pin, warp < NREP ? a.qg : a.kg, warp <= NREP ? a.qk_norm : 0, a.freq,
                       warp <= NREP ? a.rope_pairs : 0, a.pos, lane);
    if (warp != kDecodeConsumerWarps) {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    }
    if (first_job)
        head_load<D>(pin, warp < NREP ? a.q + static_cast<size_t>(g * NREP + warp) * D
                                      : (warp == NREP ? a.k : a.v) + static_cast<size_t>(g) * D, lane);

    // ------------------------------------------------------------------ producer warp
    if (warp == kDecodeConsumerWarps) {
        if (lane == 0) {
            int it = 0;        // stage uses so far
            int issued = 0;    // stage uses that carry copies
            bool fail = false;
            int base = split * a.chunk;  // first chunk: static
            const int first_dyn = a.n_split * a.chunk;
            auto issue = [&](int t, int s) {
                tile_id_s[s] = t;
                const int row = a.row0 + t * TP;
                uint8_t* kdst = tiles + s * Sm::kStageBytes;
                mbar_arrive_expect_tx(&full_k[s], kDecodeTileBytes);
                tma_load_3d(kdst, &tm_k, &full_k[s], 0, g, row);
                mbar_arrive_expect_tx(&full_v[s], kDecodeTileBytes);
                tma_load_3d(kdst + kDecodeTileBytes, &tm_v, &full_v[s], 0, g, row);
                ++issued;
            };
            // While the previous grid finishes: the first tiles of the static chunk that lie wholly
            // below a.pre_rows.  The host sets pre_rows below every row its most recent cache write
            // touched in this layer, and with programmatic launches only the immediately preceding
            // kernel can still be running (each of this library's kernels waits for its own
            // predecessor before it lets its dependent launch).
            int t0 = base;
            const int lim0 = min(base + a.chunk, a.n_tiles);
            for (; t0 < lim0 && it < kDecodeEarlyTiles && (t0 + 1) * TP <= a.pre_rows; ++t0, ++it) issue(t0, it);
            asm volatile("griddepcontrol.wait;" ::: "memory");
            bool first = true;
            while (!fail && base < a.n_tiles) {
                const int lim = min(base + a.chunk, a.n_tiles);
                int next = a.dynamic ? lim : a.n_tiles;
                int t = base;
                if (first && t0 > base) {  // part of the first chunk is already on its way
                    t = t0;
                    if (a.dynamic) next = first_dyn + atomicAdd(&a.chunk_ctr[g], a.chunk);
                }
                first = false;
                for (; t < lim; ++t, ++it) {
                    const int s = it % kDecodeStages;
                    if (it >= kDecodeStages &&
                        !mbar_wait_bounded(&empty[s], ((it / kDecodeStages) - 1) & 1, deadline, abort_s)) {
                        *abort_s = 1;
                        *reinterpret_cast<volatile int*>(a.err) = KERR_TIMEOUT_EMPTY;
                        fail = true;
                        break;
                    }
                    issue(t, s);
                    // Fetch the next chunk once this chunk's first copy is on its way: the grab's
                    // latency overlaps the remaining waits and copies instead of delaying them.
                    if (t == base && a.dynamic) next = first_dyn + atomicAdd(&a.chunk_ctr[g], a.chunk);
                }
                base = next;
            }
            bool marker = false;
            if (!fail) {  // end marker: a stage whose K barrier completes without data
                const int s = it % kDecodeStages;
                if (it >= kDecodeStages &&
                    !mbar_wait_bounded(&empty[s], ((it / kDecodeStages) - 1) & 1, deadline, abort_s)) {
                    *abort_s = 1;
                    *reinterpret_cast<volatile int*>(a.err) = KERR_TIMEOUT_EMPTY;
                } else {
                    tile_id_s[s] = -1;
                    mbar_arrive(&full_k[s]);
                    marker = true;
                }
            }
            // Our copies must land before this CTA may exit: wait for the uses not yet known to be
            // consumed (ignoring the abort flag, bounded by a later deadline).  When the end marker
            // went in, its stage's previous use was consumed (we waited on its empty barrier) and
            // that stage's K barrier is one phase ahead, so the drain starts one use later.
            const uint64_t drain_deadline = deadline + kWaitLimitNs / 2;
            for (int u = max(0, issued - kDecodeStages + (marker ? 1 : 0)); u < issued; ++u) {
                const int s = u % kDecodeStages;
                const uint32_t par = (u / kDecodeStages) & 1;
                while (!mbar_try_wait(&full_k[s], par) && globaltimer_ns() < drain_deadline) {
                }
                while (!mbar_try_wait(&full_v[s], par) && globaltimer_ns() < drain_deadline) {
                }
            }
        }
        return;
    }

    // ------------------------------------------------------------------ consumers: prologue
    {
        for (int job = warp; job < njobs; job += kDecodeConsumerWarps) {
            if (job == warp) {  // first round: inputs already in registers
                float* dst = job < NREP ? q_s + job * D : (job == NREP ? kn_s : vn_s);
                head_finish<D>(pin, job <= NREP ? a.qk_norm : 0, a.eps, job <= NREP ? a.rope_pairs : 0, dst, lane);
            } else if (job < NREP) {
                const int hq = g * NREP + job;
                norm_rope_head<D>(a.q + static_cast<size_t>(hq) * D, a.qg, a.qk_norm, a.eps, a.freq,
                                  a.rope_pairs, a.pos, q_s + job * D, lane);
            } else if (job == NREP) {
                norm_rope_head<D>(a.k + static_cast<size_t>(g) * D, a.kg, a.qk_norm, a.eps, a.freq,
                                  a.rope_pairs, a.pos, kn_s, lane);
            } else {
                for (int d = lane; d < D; d += 32) vn_s[d] = a.v[static_cast<size_t>(g) * D + d];
            }
        }
    }
    named_bar_sync(1, kDecodeConsumers);
    if (owner) {
        KV* krow = reinterpret_cast<KV*>(a.kc) + static_cast<size_t>(a.pos) * a.kv_dim + g * D;
        KV* vrow = reinterpret_cast<KV*>(a.vc) + static_cast<size_t>(a.pos) * a.kv_dim + g * D;
        for (int d = tid; d < D; d += kDecodeConsumers) {
            krow[d] = KvTraits<KV>::from_float(kn_s[d]);
            vrow[d] = KvTraits<KV>::from_float(vn_s[d]);
        }
        if (tid == 0 && a.shadow_wm) atomicMin(a.shadow_wm, a.pos);
    }

    const int r = lane / LPR, j = lane % LPR;
    float qr[NREP][EPL];
#pragma unroll
    for (int h = 0; h < NREP; ++h)
#pragma unroll
        for (int e = 0; e < EPL; ++e) qr[h][e] = q_s[h * D + j * EPL + e];

    float acc[NREP][EPL];
#pragma unroll
    for (int h = 0; h < NREP; ++h)
#pragma unroll
        for (int e = 0; e < EPL; ++e) acc[h][e] = 0.f;
    bool ok = true;
    const bool div = a.scale_div != 0;
    const float scale = a.scale;
    // Each warp consumes its own R rows of every tile (rows [warp*R, warp*R + R)) and keeps its own
    // online softmax: the running max and sum of each head over the rows it has seen.  The warps
    // never wait for one another inside the loop; their (max, sum, o) are combined once, below.
    // Softmax items: (head h, local row lr) = q = h*R + lr; lane takes q = lane + 32k, so the R items
    // of a head sit on an aligned group of R lanes (segmented shuffles), and each lane keeps the
    // running max / sum of its items' heads (replicated over the group).
    constexpr int R = NI * RPI;
    constexpr int NP = NREP * R;
    constexpr int IPL = (NP + 31) / 32;
    static_assert(R <= 32 && (R & (R - 1)) == 0, "a warp's rows form an aligned lane group");
    float* wsc = sc + warp * NREP * R;  // this warp's scores, then probabilities: [lr][h]
    float m_lane[IPL], l_lane[IPL];
#pragma unroll
    for (int k = 0; k < IPL; ++k) {
        m_lane[k] = -INFINITY;
        l_lane[k] = 0.f;
    }

    for (int it = 0;; ++it) {
        const int s = it % kDecodeStages;
        const uint32_t par = (it / kDecodeStages) & 1;
        const uint8_t* kt = tiles + s * Sm::kStageBytes;
        const uint8_t* vt = kt + kDecodeTileBytes;

        ok = __all_sync(0xffffffffu, mbar_wait_bounded(&full_k[s], par, deadline, abort_s));
        if (!ok) {
            if (lane == 0) {
                *abort_s = 1;
                *reinterpret_cast<volatile int*>(a.err) = KERR_TIMEOUT_FULL;
            }
            break;
        }
        const int tile = tile_id_s[s];  // -1: the producer's end marker
        if (tile < 0) break;
        const int tbase = tile * TP;
        {
            float part[NV];
#pragma unroll
            for (int i = 0; i < NI; ++i) {
                const int row = (warp * NI + i) * RPI + r;
                const uint4 raw = lds128(kt + row * RB + j * 16);
                float kx[EPL];
                KvTraits<KV>::unpack(raw, kx);
#pragma unroll
                for (int h = 0; h < NREP; ++h) {
                    float d0 = 0.f;
#pragma unroll
                    for (int e = 0; e < EPL; ++e) d0 = fmaf(kx[e], qr[h][e], d0);
                    part[i * NREP + h] = d0;
                }
            }
            transposed_reduce<NV, S>(part, lane);
            if constexpr (NV >= (1 << S)) {
                constexpr int VF = NV >> S;
#pragma unroll
                for (int u = 0; u < VF; ++u) {
                    const int vi = j * VF + u;
                    const int i = vi / NREP, h = vi % NREP;
                    const int lr = i * RPI + r;
                    const float sv = div ? part[u] / scale : part[u] * scale;
                    wsc[lr * NREP + h] = (tbase + (warp * NI + i) * RPI + r < t_end) ? sv : -INFINITY;
                }
            } else {
                constexpr int DUP = (1 << S) / NV;
                if (j % DUP == 0) {
                    const int vi = j / DUP;
                    const int i = vi / NREP, h = vi % NREP;
                    const int lr = i * RPI + r;
                    const float sv = div ? part[0] / scale : part[0] * scale;
                    wsc[lr * NREP + h] = (tbase + (warp * NI + i) * RPI + r < t_end) ? sv : -INFINITY;
                }
            }
        }
        __syncwarp();
        // Online softmax of this warp's rows, per head: e^x as 2^(x log2 e) on the MUFU
        // (ex2.approx, relative error about 2^-22).  The accumulators are rescaled only when some
        // head's running maximum moved (a factor of exactly 1 otherwise).
        float ck[IPL];
        bool moved = false;
#pragma unroll
        for (int k = 0; k < IPL; ++k) {
            const int q = lane + 32 * k;
            const int ws = (q % R) * NREP + q / R;  // item (head q / R, row q % R)
            const float sv = q < NP ? wsc[ws] : -INFINITY;
            float mx = sv;
#pragma unroll
            for (int o = R / 2; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float mn = fmaxf(m_lane[k], mx);
            ck[k] = mn == -INFINITY ? 1.f : decode_exp2((m_lane[k] - mn) * kLog2e);
            moved |= ck[k] != 1.f;
            const float p = mn == -INFINITY ? 0.f : decode_exp2((sv - mn) * kLog2e);
            float ps = p;
#pragma unroll
            for (int o = R / 2; o >= 1; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
            l_lane[k] = l_lane[k] * ck[k] + ps;
            m_lane[k] = mn;
            if (q < NP) wsc[ws] = p;
        }
        __syncwarp();
        ok = __all_sync(0xffffffffu, mbar_wait_bounded(&full_v[s], par, deadline, abort_s));
        if (!ok) {
            if (lane == 0) {
                *abort_s = 1;
                *reinterpret_cast<volatile int*>(a.err) = KERR_TIMEOUT_FULL;
            }
            break;
        }
        if (__any_sync(0xffffffffu, moved)) {
#pragma unroll
            for (int h = 0; h < NREP; ++h) {
                const float c = __shfl_sync(0xffffffffu, ck[(h * R) / 32], (h * R) % 32);
#pragma unroll
                for (int e = 0; e < EPL; ++e) acc[h][e] *= c;
            }
        }
#pragma unroll
        for (int i = 0; i < NI; ++i) {
            const int row = (warp * NI + i) * RPI + r;
            const uint4 raw = lds128(vt + row * RB + j * 16);
            if (tbase + row < t_end) {
                float vx[EPL];
                KvTraits<KV>::unpack(raw, vx);
                float pv[NREP];  // the row's probabilities for every head, one vector load
                const float* pr = wsc + (i * RPI + r) * NREP;
                if constexpr (NREP % 4 == 0) {
#pragma unroll
                    for (int c = 0; c < NREP / 4; ++c) {
                        const float4 t4 = reinterpret_cast<const float4*>(pr)[c];
                        pv[4 * c] = t4.x;
                        pv[4 * c + 1] = t4.y;
                        pv[4 * c + 2] = t4.z;
                        pv[4 * c + 3] = t4.w;
                    }
                } else if constexpr (NREP == 2) {
                    const float2 t2 = *reinterpret_cast<const float2*>(pr);
                    pv[0] = t2.x;
                    pv[1] = t2.y;
                } else {
                    pv[0] = pr[0];
                }
#pragma unroll
                for (int h = 0; h < NREP; ++h)
#pragma unroll
                    for (int e = 0; e < EPL; ++e) acc[h][e] = fmaf(pv[h], vx[e], acc[h][e]);
            }
        }
        __syncwarp();  // every lane is done with this stage and with wsc
        if (lane == 0) mbar_arrive(&empty[s]);
    }

    // ------------------------------------------------------------------ CTA reduction
    // Warp w holds (m_w, l_w, o_w) per head over its rows; with M = max_w m_w the CTA's result is
    // o = sum_w o_w e^(m_w - M), l = sum_w l_w e^(m_w - M), m = M.
#pragma unroll
    for (int o = LPR; o < 32; o <<= 1)
#pragma unroll
        for (int h = 0; h < NREP; ++h)
#pragma unroll
            for (int e = 0; e < EPL; ++e) acc[h][e] += __shfl_xor_sync(0xffffffffu, acc[h][e], o);
    float mh[NREP], lh[NREP];
#pragma unroll
    for (int h = 0; h < NREP; ++h) {
        mh[h] = __shfl_sync(0xffffffffu, m_lane[(h * R) / 32], (h * R) % 32);
        lh[h] = __shfl_sync(0xffffffffu, l_lane[(h * R) / 32], (h * R) % 32);
    }
    named_bar_sync(1, kDecodeConsumers);  // every warp is done with the tiles before `red` aliases them
    float* red = reinterpret_cast<float*>(tiles);                       // [warp][NREP][D]
    float* wml = red + kDecodeConsumerWarps * NREP * D;                 // [warp][2][NREP]
    if (lane < LPR) {
#pragma unroll
        for (int h = 0; h < NREP; ++h)
#pragma unroll
            for (int e = 0; e < EPL; ++e) red[(warp * NREP + h) * D + j * EPL + e] = acc[h][e];
    }
    if (lane == 0) {
#pragma unroll
        for (int h = 0; h < NREP; ++h) {
            wml[(warp * 2) * NREP + h] = mh[h];
            wml[(warp * 2 + 1) * NREP + h] = lh[h];
        }
    }
    named_bar_sync(1, kDecodeConsumers);
    for (int idx = tid; idx < NREP * D; idx += kDecodeConsumers) {
        const int h = idx / D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kDecodeConsumerWarps; ++w) M = fmaxf(M, wml[(w * 2) * NREP + h]);
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < kDecodeConsumerWarps; ++w) {
            const float mw = wml[(w * 2) * NREP + h];
            if (mw != -INFINITY) sum = fmaf(red[w * NREP * D + idx], expf(mw - M), sum);
        }
        o_s[idx] = sum;
    }
    if (tid < NREP) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kDecodeConsumerWarps; ++w) M = fmaxf(M, wml[(w * 2) * NREP + tid]);
        float L = 0.f;
#pragma unroll
        for (int w = 0; w < kDecodeConsumerWarps; ++w) {
            const float mw = wml[(w * 2) * NREP + tid];
            if (mw != -INFINITY) L = fmaf(wml[(w * 2 + 1) * NREP + tid], expf(mw - M), L);
        }
        m_s[tid] = M;
        l_s[tid] = L;
    }
    named_bar_sync(1, kDecodeConsumers);

    // ------------------------------------------------------------------ current token (t == pos)
    if (owner) {
        if (warp < NREP) {
            const int h = warp;
            float d0 = 0.f;
            for (int d = lane; d < D; d += 32) d0 = fmaf(q_s[h * D + d], kn_s[d], d0);
            d0 = warp_sum(d0);
            const float sv = div ? d0 / scale : d0 * scale;
            const float m_old = m_s[h];
            const float m_new = fmaxf(m_old, sv);
            const float ca = expf(m_old - m_new), cb = expf(sv - m_new);
            for (int d = lane; d < D; d += 32) o_s[h * D + d] = o_s[h * D + d] * ca + cb * vn_s[d];
            __syncwarp();
            if (lane == 0) {
                m_s[h] = m_new;
                l_s[h] = l_s[h] * ca + cb;
            }
        }
        named_bar_sync(1, kDecodeConsumers);
    }
    if (tid == 0) *stop_s = *abort_s;
    named_bar_sync(1, kDecodeConsumers);
    if (*stop_s) return;

    const int head0 = g * NREP;
    int grp_out = 0, n_out = 1;  // gather: the group this CTA's words carry, of how many (1: the output)
    if (a.n_split > 1) {
        // Two-level merge: the last CTA of each group of a.merge_group splits merges the group,
        // then (with more than one group) the last group merger merges the group results.  A
        // gathered decode with at most kGatherGroups groups skips the second level: each group
        // merger stores its group's result and the gather wait of every rank merges them.
        constexpr int PS = decode_part_stride(NREP, D);
        const int GRP = a.merge_group;  // <= Sm::kMergeGroup, so that a group's copy fits the ring
        const int kvh = a.kv_dim / D;
        float* pp = a.part + (static_cast<size_t>(g) * kDecodeMaxSplit + split) * PS;
        for (int idx = tid; idx < NREP * D; idx += kDecodeConsumers) pp[idx] = o_s[idx];
        if (tid < NREP) {
            pp[NREP * D + tid] = m_s[tid];
            pp[NREP * D + NREP + tid] = l_s[tid];
        }
        named_bar_sync(1, kDecodeConsumers);
        const int grp = split / GRP;
        const int n_groups = (a.n_split + GRP - 1) / GRP;
        const int gsize = min(GRP, a.n_split - grp * GRP);
        int* grp_ctr = a.counters + 2 * kvh + g * kDecodeMaxGroups + grp;
        if (tid == 0) *last_s = (ticket_acq_rel(grp_ctr) == gsize - 1) ? 1 : 0;
        named_bar_sync(1, kDecodeConsumers);
        if (!*last_s) return;
        // The tiles are free: the merge copies the partials there; its weights go to the score buffer.
        if (!merge_partials<NREP, D>(a.part + (static_cast<size_t>(g) * kDecodeMaxSplit + grp * GRP) * PS, gsize,
                                     tiles, sc, merge_bar, 0, o_s, m_s, l_s, tid, warp, lane, deadline, abort_s,
                                     a.err))
            return;
        if (tid == 0) *grp_ctr = 0;
        if (a.peer_ll && n_groups > 1 && n_groups <= kGatherGroups) {
            grp_out = grp;
            n_out = n_groups;
            // With grabs, the last group merger of the head (head ticket) frees the grab counter:
            // every CTA of the head took its group ticket after its last grab.
            if (a.dynamic) {
                if (tid == 0) *last_s = (ticket_acq_rel(&a.counters[g]) == n_groups - 1) ? 1 : 0;
                named_bar_sync(1, kDecodeConsumers);
                if (tid == 0 && *last_s) {
                    a.counters[g] = 0;
                    a.chunk_ctr[g] = 0;
                }
            }
        } else {
            if (n_groups > 1) {
                float* gp = a.gpart + (static_cast<size_t>(g) * kDecodeMaxGroups + grp) * PS;
                for (int idx = tid; idx < NREP * D; idx += kDecodeConsumers) gp[idx] = o_s[idx];
                if (tid < NREP) {
                    gp[NREP * D + tid] = m_s[tid];
                    gp[NREP * D + NREP + tid] = l_s[tid];
                }
                named_bar_sync(1, kDecodeConsumers);
                if (tid == 0) *last_s = (ticket_acq_rel(&a.counters[g]) == n_groups - 1) ? 1 : 0;
                named_bar_sync(1, kDecodeConsumers);
                if (!*last_s) return;
                if (!merge_partials<NREP, D>(a.gpart + static_cast<size_t>(g) * kDecodeMaxGroups * PS, n_groups,
                                             tiles, sc, merge_bar, 1, o_s, m_s, l_s, tid, warp, lane, deadline,
                                             abort_s, a.err))
                    return;
                if (tid == 0) a.counters[g] = 0;
            }
            // Every CTA of this head took its group ticket after its last grab: the counter is free.
            if (tid == 0) a.chunk_ctr[g] = 0;
        }
    }
    if (a.peer_ll) {
        // The next layer's decode may start once the gathered words have arrived, before this grid
        // has completed: the counter resets above go out before any word does.
        if (a.n_split > 1) {
            __threadfence();
            named_bar_sync(1, kDecodeConsumers);
        }
        // Multi-GPU gather: every value goes to every rank's gather slot as one 64-bit word,
        // (epoch << 32) | fp32 bits, stored with a single relaxed system-scope store.  A reader that
        // sees the current epoch in a word has that word's value: no fence, no flags.
        // The epoch lives in device memory (the gather wait of the previous call advanced it), so a
        // captured CUDA graph replays correctly.  Two consecutive elements per 16-byte store.  One
        // group: the normalised output; several: this group's o (unnormalised), m and l.  Each head's
        // count word tells the readers which.
        const int epoch = __ldcg(a.epoch) + 1;
        unsigned long long* const* peers = a.peer_ll + (epoch & 1) * a.nranks;
        const unsigned long long tag = static_cast<unsigned long long>(static_cast<uint32_t>(epoch)) << 32;
        const size_t vec = static_cast<size_t>(a.g_heads) * D;
        const size_t obase = static_cast<size_t>(grp_out) * vec + a.q_off + static_cast<size_t>(head0) * D;
        for (int idx = 2 * tid; idx < NREP * D; idx += 2 * kDecodeConsumers) {
            const float v0 = n_out == 1 ? o_s[idx] / l_s[idx / D] : o_s[idx];
            const float v1 = n_out == 1 ? o_s[idx + 1] / l_s[(idx + 1) / D] : o_s[idx + 1];
            const unsigned long long w0 = tag | __float_as_uint(v0);
            const unsigned long long w1 = tag | __float_as_uint(v1);
            for (int rr = 0; rr < a.nranks; ++rr)
                asm volatile("st.relaxed.sys.global.v2.b64 [%0], {%1, %2};" ::"l"(peers[rr] + obase + idx), "l"(w0),
                             "l"(w1)
                             : "memory");
        }
        if (tid < NREP) {
            const size_t qh = static_cast<size_t>(a.q_off / D + head0 + tid);  // global q head
            const size_t mo = gather_m_off(a.g_heads, D) + static_cast<size_t>(grp_out) * a.g_heads + qh;
            const size_t lo = gather_l_off(a.g_heads, D) + static_cast<size_t>(grp_out) * a.g_heads + qh;
            const size_t co = gather_cnt_off(a.g_heads, D) + qh;
            const unsigned long long wm = tag | __float_as_uint(m_s[tid]);
            const unsigned long long wl = tag | __float_as_uint(l_s[tid]);
            const unsigned long long wc = tag | static_cast<uint32_t>(n_out);
            for (int rr = 0; rr < a.nranks; ++rr) {
                if (n_out > 1) {
                    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(peers[rr] + mo), "l"(wm) : "memory");
                    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(peers[rr] + lo), "l"(wl) : "memory");
                }
                asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(peers[rr] + co), "l"(wc) : "memory");
            }
        }
        return;
    }
    for (int idx = tid; idx < NREP * D; idx += kDecodeConsumers)
        a.out[static_cast<size_t>(head0) * D + idx] = o_s[idx] / l_s[idx / D];
}

}  // namespace lg
