// flash_tc.cuh - bf16 tensor-core attention (tcgen05 + TMEM + TMA) for causal prefill and BERT.
//
// Same semantics as flash_simt.cuh (prefill = the reference's one-token-at-a-time loop,
// fast/ligguf_fast_qk.cpp:340-356; BERT = fast/vdb.cpp:189-212 per sequence), with q, k, v rounded
// to bf16 and every product accumulated in fp32 by the tensor cores.
//
// Work item = 128 query rows (one tile) of one q head of one batch entry.  A kernel that uses
// tcgen05 runs one CTA per SM, so the grid is persistent: one CTA per SM walks a fixed share of the
// items, keeping its barriers and all 512 TMEM columns across them, and the overlap of tensor-core
// work with softmax work comes from inside the CTA (512 threads, four warpgroups whose register
// budgets are rebalanced with setmaxnreg):
//   warp 0      TMA producer: per item the Q tile (double-buffered), then K and V tiles of 128 keys
//               into 2-stage rings (3 for D = 64)
//   warp 1      allocates TMEM; lane 0 issues S = Q.K^T: D/16 MMAs of M128 N128 K16 per tile, Q and
//               K from shared memory (K-major, SWIZZLE_128B)
//   warp 2      lane 0 issues O += P.V: 8 MMAs of M128 N=D K16 per tile, P from TMEM, V from shared
//               memory (MN-major, SWIZZLE_128B)
//   warp 3      idle (completes the first warpgroup)
//   warps 4..11 softmax, two threads per query row (= TMEM lane): warps 4-7 take S columns
//               [0, 64), warps 8-11 columns [64, 128) of the same lanes; each reads its half of the
//               row from TMEM once into registers, the two exchange their half maxima through
//               shared memory, then each writes its P half as bf16 pairs back into TMEM, rescales
//               its half of O when the running max moves (rare), and keeps its half of the row sum
//   warps 12..15 epilogue: O / l from TMEM to global memory through a padded staging block (whole
//               128-byte row segments per store), so the softmax warps never wait for it
// Items are walked heaviest first: causal prefill by their numbering, BERT through a work order
// sorted by key-tile count that the operand conversion kernel writes (bert_item_order).
// TMEM: S double buffer [0, 256), O double-buffered by item after it.  An issuing thread loses
// issue slots to the softmax warp on its SM sub-partition, so S and P.V are issued by two threads
// on different sub-partitions, and tiles are 128 keys wide to halve the MMAs and barrier waits per
// key.  MMAs of different threads are not ordered: S(t+2), which overwrites the buffer that P(t) was
// packed into, waits for P.V(t) to complete (pv_done).  Every wait is bounded; on a timeout the
// kernel records an error, drains its own copies and MMAs, frees TMEM and returns.
#pragma once

#include "common.cuh"

namespace lg {

struct TcArgs {
    const __nv_bfloat16* q;  // [q_rows][q_heads][D]
    const __nv_bfloat16* k;  // [kv_rows][kv_heads][D]
    const __nv_bfloat16* v;
    float* out;              // [q_rows][q_heads][D]
    int q_rows, q_heads, kv_rows, kv_heads;
    int batch, q_seq, kv_seq;  // batch entry b owns rows [b*q_seq, b*q_seq + len_b)
    const int* lens;           // per-batch valid rows (or null: q_seq / kv_seq)
    int causal, q_pos0, nrep;
    float scale_log2;          // softmax scale times log2(e)
    int* err;
    const int* order;  // null, or order[p] = the item taken at walk position p (a permutation)
};

constexpr int kTcRows = 128;  // query rows per tile (UMMA M)
constexpr int kTcKeys = 128;  // keys per tile (UMMA N of S, K of P.V)

// Work order for a BERT batch.  The items (head, query tile, batch entry; numbered as in tc_item)
// are sorted by their number of key tiles, most first, so that the persistent CTAs' snake walk
// (tc_item_index) deals out even shares whatever the sequence lengths: with lengths in the walk's
// natural order the busiest CTA gets 14-39 % more key tiles than the mean on U[16, 512] lengths,
// sorted 1-4 %.  A counting sort by one block; items of equal cost land in arbitrary order
// (shared-memory atomics), which decides only which CTA computes an item, never its result.
constexpr int kOrderBins = 1025;  // key-tile counts 0..1024: max_len up to 131072
__device__ __forceinline__ int bert_group_cost(const int* lens, int g, int n_qt, int max_len) {
    const int b = g / n_qt, y = g - b * n_qt;
    const int r0 = (n_qt - 1 - y) * kTcRows;  // tc_item: y = 0 is the last query tile
    const int len = min(lens[b], max_len);
    return r0 >= len ? 0 : (len + kTcKeys - 1) / kTcKeys;
}
__device__ void bert_item_order(const int* __restrict__ lens, int batch, int max_len, int n_heads,
                                int* __restrict__ order) {
    __shared__ int bins[kOrderBins];
    const int n_qt = (max_len + kTcRows - 1) / kTcRows;
    const int top = (max_len + kTcKeys - 1) / kTcKeys;  // largest cost; the host keeps it < kOrderBins
    const int groups = n_qt * batch;                    // group g = y + n_qt * b: n_heads items each
    for (int i = threadIdx.x; i <= top; i += blockDim.x) bins[i] = 0;
    __syncthreads();
    for (int g = threadIdx.x; g < groups; g += blockDim.x)
        atomicAdd(&bins[bert_group_cost(lens, g, n_qt, max_len)], 1);
    __syncthreads();
    if (threadIdx.x == 0) {  // exclusive scan, the largest cost first
        int run = 0;
        for (int c = top; c >= 0; --c) {
            const int n = bins[c];
            bins[c] = run;
            run += n;
        }
    }
    __syncthreads();
    for (int g = threadIdx.x; g < groups; g += blockDim.x) {
        const int p = atomicAdd(&bins[bert_group_cost(lens, g, n_qt, max_len)], 1);
        for (int h = 0; h < n_heads; ++h) order[p * n_heads + h] = g * n_heads + h;
    }
}

// BERT operands to bf16 in one pass, valid rows only: rows r < lens[b] of q, k and v are converted.
// Every padded v row that some key tile reads is written as zeros (P.V multiplies it by P = 0, and
// 0 * NaN is NaN, so it must be finite whatever the buffer held before): the rows inside this
// entry's last key tile that holds valid keys, and - when max_len is not a multiple of the tile -
// the first rows of this entry that the previous entry's last tile runs into.  The tensor-core
// kernel reads no other padded row.  Padded rows of q and k are left as they are (their scores are
// masked or their outputs discarded).
// Block = kBertConvRows rows of one batch entry; 8 values per thread step (two 16-byte loads, one
// 16-byte store).  Needs E % 8 == 0 and 16-byte aligned bases.  With `order` set, the grid has one
// more column of blocks, and its first block writes the work order (bert_item_order) instead.
constexpr int kBertConvRows = 8;
__global__ void __launch_bounds__(256) bert_to_bf16_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                                           const float* __restrict__ v, const int* __restrict__ lens,
                                                           int max_len, int E, __nv_bfloat16* __restrict__ bq,
                                                           __nv_bfloat16* __restrict__ bk, __nv_bfloat16* __restrict__ bv,
                                                           int n_heads, int* __restrict__ order) {
    // Launched in stream order (its predecessor has completed); the tensor-core kernel that follows
    // is a programmatic dependent and may start its set-up once every block of this grid has begun.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (order && blockIdx.x == gridDim.x - 1) {
        if (blockIdx.y == 0) bert_item_order(lens, gridDim.y, max_len, n_heads, order);
        return;
    }
    const int b = blockIdx.y;
    const int r0 = blockIdx.x * kBertConvRows;
    const int len = min(lens[b], max_len);
    // Key tiles of entry b start at multiples of kTcKeys from its first row, so its last tile may
    // run up to round_up(max_len) - max_len rows into entry b + 1.
    const int tile_end = (len + kTcKeys - 1) / kTcKeys * kTcKeys;
    const int overhang = b > 0 ? (max_len + kTcKeys - 1) / kTcKeys * kTcKeys - max_len : 0;
    const int v_zero_end = min(max_len, max(tile_end, overhang));
    const int units = E / 8;  // 16-byte output units per row
    const int per_tensor = kBertConvRows * units;
    for (int u = threadIdx.x; u < 3 * per_tensor; u += blockDim.x) {
        const int t = u / per_tensor;
        const int rem = u - t * per_tensor;
        const int r = r0 + rem / units;
        if (r >= max_len) continue;
        const size_t off = (static_cast<size_t>(b) * max_len + r) * E + size_t(rem % units) * 8;
        __nv_bfloat16* dst = t == 0 ? bq : (t == 1 ? bk : bv);
        if (r >= len) {
            if (t == 2 && r < v_zero_end) *reinterpret_cast<uint4*>(dst + off) = make_uint4(0u, 0u, 0u, 0u);
            continue;
        }
        const float* src = t == 0 ? q : (t == 1 ? k : v);
        const float4 x0 = __ldcs(reinterpret_cast<const float4*>(src + off));
        const float4 x1 = __ldcs(reinterpret_cast<const float4*>(src + off) + 1);
        const __nv_bfloat162 p0 = __floats2bfloat162_rn(x0.x, x0.y), p1 = __floats2bfloat162_rn(x0.z, x0.w);
        const __nv_bfloat162 p2 = __floats2bfloat162_rn(x1.x, x1.y), p3 = __floats2bfloat162_rn(x1.z, x1.w);
        *reinterpret_cast<uint4*>(dst + off) =
            make_uint4(*reinterpret_cast<const uint32_t*>(&p0), *reinterpret_cast<const uint32_t*>(&p1),
                       *reinterpret_cast<const uint32_t*>(&p2), *reinterpret_cast<const uint32_t*>(&p3));
    }
}

// Four warpgroups: 0 = TMA producer (warp 0), S issuer (warp 1), P.V issuer (warp 2), warp 3 idle;
// 1 and 2 = softmax, column halves of every row (warps 4-7, 8-11); 3 = epilogue (warps 12-15).  A
// warp reaches only TMEM lanes [32 * (warp % 4), +32), so each of the last three warpgroups covers
// all 128 lanes.
constexpr int kTcThreads = 512;
constexpr int kTcPvWarp = 2;  // the warp that issues the P.V MMAs
// Register split (setmaxnreg) from the 128 per thread that 512 threads at one CTA per SM launch with:
// a softmax thread holds half of a 128-column S row in registers, an epilogue thread a 32-column
// block of O.  The sum of the four shares must not exceed 4 x 128, or an increase waits forever; the
// launcher checks the kernel's register count.  (This split compiles without spills.)
constexpr int kTcRegsLaunch = 128;
constexpr int kTcRegsIssue = 56;
constexpr int kTcRegsSoftmax = 160;
constexpr int kTcRegsEpilogue = 136;
static_assert(kTcRegsIssue + 2 * kTcRegsSoftmax + kTcRegsEpilogue <= 4 * kTcRegsLaunch, "register split too large");
static_assert(kTcThreads * kTcRegsLaunch <= 65536, "launch register count does not fit an SM");
// A kernel that uses tcgen05 runs one CTA per SM, which then owns all 512 TMEM columns:
// S double buffer [0, 256) (P of a tile is packed over the first 64 columns of its S buffer),
// O double buffer (by item) [256, 256 + 2D).
constexpr uint32_t kTcTmemCols = 512;
template <int D>
struct TcTmem {
    static constexpr uint32_t kS = 0;
    static constexpr uint32_t kO = 2 * kTcKeys;
    static_assert(kO + 2 * D <= kTcTmemCols, "TMEM plan exceeds 512 columns");
};

template <int D>
struct TcSmem {
    static constexpr int kChunks = D / 64;               // 128-byte column chunks of a row
    static constexpr int kQBytes = kTcRows * D * 2;      // a Q tile: 128 rows of bf16
    static constexpr int kQChunkBytes = kTcRows * 128;   // one 128-byte-wide chunk of a Q tile
    static constexpr int kKvBytes = kTcKeys * D * 2;     // a K or V tile: 128 rows of bf16
    static constexpr int kKvChunkBytes = kTcKeys * 128;  // one 128-byte-wide chunk of a K/V tile
    // K/V ring: 128 KB for D 128; 96 KB for D 64, where 3 stages measured faster than 2, 4 or 5.
    static constexpr int kStages = D == 128 ? 2 : 3;
    static constexpr int kLRing = 4;                     // row-sum slots (by item)
    static constexpr size_t kQ = 0;                      // Q double buffer (by item)
    static constexpr size_t kK = kQ + 2 * size_t(kQBytes);
    static constexpr size_t kV = kK + size_t(kStages) * kKvBytes;
    static constexpr size_t kL = kV + size_t(kStages) * kKvBytes;  // row sums l, [kLRing][2 halves][128] fp32
    // Epilogue staging: per epilogue warp a 32 x 32 fp32 block, rows padded to 36 floats (16-byte
    // aligned, conflict-free float4 accesses both ways).
    static constexpr int kStageRow = 36;
    static constexpr size_t kX = kL + size_t(kLRing) * 2 * kTcRows * 4;  // half-row maxima [2 tiles][2][128]
    static constexpr size_t kE = kX + size_t(2) * 2 * kTcRows * 4;
    static constexpr size_t kBar = kE + 4 * 32 * kStageRow * 4;
    // k_full[S], k_empty[S], v_full[S], v_empty[S], s_full[2], p_full[2], pv_done[2], drain, q_full[2],
    // q_empty[2], o_final[2], o_free[2], l_full[kLRing]
    static constexpr int kNumBars = 4 * kStages + 2 + 2 + 2 + 1 + 8 + kLRing + 8;  // + xchg[2][4]
    static constexpr size_t kMisc = kBar + size_t(kNumBars) * 8;  // tmem base, abort flag
    static constexpr size_t kTotal = kMisc + 16 + 1024;           // + slack to align the base to 1 KB
};

// ------------------------------------------------------------------------------ tcgen05 wrappers
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (bf16 inputs, fp32 accumulate), cta_group::1.
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]: A (M x 16, bf16 pairs packed in 32-bit columns) from TMEM.
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrives once on `bar` when every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// Shared-memory matrix descriptor, SWIZZLE_128B (sm100 layout code 2, descriptor version 1).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return uint64_t((saddr >> 4) & 0x3FFFu) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
           (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46) | (uint64_t(2) << 61);
}
// The same descriptor `bytes` further on: the start address is the low 14-bit field (address >> 4),
// and shared-memory addresses stay below 2^18, so the add never carries out of the field.
__device__ __forceinline__ uint64_t desc_advance(uint64_t desc, uint32_t bytes) { return desc + (bytes >> 4); }
// Instruction descriptor, kind::f16: bf16 A and B, fp32 accumulator, M x N, majors (0 K, 1 MN).
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, int a_mn, int b_mn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(a_mn) << 15) | (uint32_t(b_mn) << 16) |
           (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

#define LG_R32(p) \
    "=r"(p[0]), "=r"(p[1]), "=r"(p[2]), "=r"(p[3]), "=r"(p[4]), "=r"(p[5]), "=r"(p[6]), "=r"(p[7]), \
    "=r"(p[8]), "=r"(p[9]), "=r"(p[10]), "=r"(p[11]), "=r"(p[12]), "=r"(p[13]), "=r"(p[14]), "=r"(p[15]), \
    "=r"(p[16]), "=r"(p[17]), "=r"(p[18]), "=r"(p[19]), "=r"(p[20]), "=r"(p[21]), "=r"(p[22]), "=r"(p[23]), \
    "=r"(p[24]), "=r"(p[25]), "=r"(p[26]), "=r"(p[27]), "=r"(p[28]), "=r"(p[29]), "=r"(p[30]), "=r"(p[31])
#define LG_W32(p) \
    "r"(p[0]), "r"(p[1]), "r"(p[2]), "r"(p[3]), "r"(p[4]), "r"(p[5]), "r"(p[6]), "r"(p[7]), "r"(p[8]), \
    "r"(p[9]), "r"(p[10]), "r"(p[11]), "r"(p[12]), "r"(p[13]), "r"(p[14]), "r"(p[15]), "r"(p[16]), "r"(p[17]), \
    "r"(p[18]), "r"(p[19]), "r"(p[20]), "r"(p[21]), "r"(p[22]), "r"(p[23]), "r"(p[24]), "r"(p[25]), "r"(p[26]), \
    "r"(p[27]), "r"(p[28]), "r"(p[29]), "r"(p[30]), "r"(p[31])

// 32 consecutive fp32 columns of this thread's TMEM lane (warp-collective, 32x32b shape).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : LG_R32(r)
        : "r"(taddr)
        : "memory");
}
// Same, into 32 consecutive elements of a larger register array (no wait: batch several, then
// tmem_wait_ld once).
__device__ __forceinline__ void tmem_ld32p(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : LG_R32(r)
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
            taddr),
        LG_W32(r)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}
__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
                 : "memory");
}

// Waits bounded; on failure records `code`, raises the CTA abort flag and returns false.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, uint64_t deadline, volatile int* abort,
                                        int* err, int code) {
    if (mbar_wait_bounded(bar, parity, deadline, abort)) return true;
    *abort = 1;
    *reinterpret_cast<volatile int*>(err) = code;
    return false;
}

// Packed fp32 pair arithmetic (sm_100 f32x2 instructions): half the issue slots of two scalar ops.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "add.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
// Warpgroup-wide register budget change (all 128 threads of the warpgroup execute it together).
template <int R>
__device__ __forceinline__ void reg_dec() {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(R));
}
template <int R>
__device__ __forceinline__ void reg_inc() {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(R));
}
// A warpgroup's share R set from the launch count: an increase or a decrease, chosen at compile time
// (.dec to a count above the current one, or .inc below it, is an illegal instruction).
template <int R>
__device__ __forceinline__ void reg_set() {
    static_assert(R % 8 == 0 && R >= 24 && R <= 256, "setmaxnreg takes a multiple of 8 in [24, 256]");
    if constexpr (R > kTcRegsLaunch)
        reg_inc<R>();
    else if constexpr (R < kTcRegsLaunch)
        reg_dec<R>();
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// 2^x for a pair, on the FMA pipe instead of the MUFU unit, which the softmax otherwise saturates:
// Cody-Waite reduction x = n + f (n = x rounded to an integer by adding 1.5 * 2^23, |f| <= 1/2),
// 2^f from a cubic p(f) = 1 + f (c1 + f (c2 + f c3)) fitted to 2^f on [-1/2, 1/2] by minimax-
// weighted least squares (max relative error 1.03e-4, below the 2^-9 rounding of P to bf16), and
// 2^n added into the exponent field.  x <= -127 gives 0 (x is clamped there: n = -127, f = 0);
// -126 > x > -127 gives a value below 2^-126 that is not exact, and bf16 P then holds zero or a
// subnormal either way.  The softmax's x never exceeds +8.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
    x.x = fmaxf(x.x, -127.f);
    x.y = fmaxf(x.y, -127.f);
    const float2 t = fadd2(x, make_float2(12582912.f, 12582912.f));  // 1.5 * 2^23 + n
    const float2 n = fadd2(t, make_float2(-12582912.f, -12582912.f));
    const float2 f = ffma2(n, make_float2(-1.f, -1.f), x);
    float2 p = ffma2(f, make_float2(0.05500665679574013f, 0.05500665679574013f),
                     make_float2(0.24220559000968933f, 0.24220559000968933f));
    p = ffma2(p, f, make_float2(0.6932826042175293f, 0.6932826042175293f));
    p = ffma2(p, f, make_float2(1.f, 1.f));
    // The low 9 bits of t's pattern hold n (two's complement); shifted into the exponent field they
    // add n to p's exponent (the bits above wrap out of the word).
    return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
                       __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
}
// Key pairs (c mod 8, in a row's 64 pairs) whose exp2 takes the polynomial: 2 of 8 (a quarter of
// the elements).  Measured: a quarter beats none, three eighths and a half.
constexpr unsigned kTcPolyPairs = 0x88u;

// One work item: 128 query rows (one tile) of one head of one batch entry.  n_kv == 0 marks an item
// of padded query rows only, which is written as zeros and never reaches the tensor cores.
struct TcItem {
    int h, b, r0, nq_valid, kv_len, n_kv;
};
// Items are numbered head fastest, then query tile from the last (longest under the causal mask)
// to the first, then batch entry, so that the heaviest items come first.
__device__ __forceinline__ TcItem tc_item(const TcArgs& a, int idx, int n_qt) {
    TcItem it;
    it.h = idx % a.q_heads;
    const int y = (idx / a.q_heads) % n_qt;
    it.b = idx / (a.q_heads * n_qt);
    it.r0 = (n_qt - 1 - y) * kTcRows;
    it.nq_valid = a.lens ? min(a.lens[it.b], a.q_seq) : a.q_seq;
    it.kv_len = a.lens ? min(a.lens[it.b], a.kv_seq) : a.kv_seq;
    int kv_eff = it.kv_len;
    if (a.causal) kv_eff = min(kv_eff, a.q_pos0 + min(it.r0 + kTcRows, it.nq_valid));
    it.n_kv = it.r0 >= it.nq_valid ? 0 : max(0, (kv_eff + kTcKeys - 1) / kTcKeys);
    return it;
}
// The w-th item of this CTA.  The grid is persistent (as many CTAs as fit at once) and walks the
// items in waves of gridDim.x, every other wave in reverse CTA order: with the heaviest items
// first, the CTA that took the heaviest item of one wave takes the lightest of the next.
__device__ __forceinline__ int tc_item_index(int w) {
    const int G = gridDim.x;
    return w * G + ((w & 1) ? G - 1 - static_cast<int>(blockIdx.x) : static_cast<int>(blockIdx.x));
}
// The item at walk position w of this CTA (through the work order when there is one), or -1 past
// the last item.  Every role of the CTA walks the same sequence.
__device__ __forceinline__ int tc_walk(const TcArgs& a, int w, int n_items) {
    const int p = tc_item_index(w);
    if (p >= n_items) return -1;
    return a.order ? __ldg(a.order + p) : p;
}

template <int D>
__global__ void __launch_bounds__(kTcThreads, 1)
    flash_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const TcArgs a) {
    using Sm = TcSmem<D>;
    using Tm = TcTmem<D>;
    constexpr int S = Sm::kStages;
    constexpr int NCH = Sm::kChunks;
    constexpr int LR = Sm::kLRing;
    extern __shared__ uint8_t tc_smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Sm::kBar);
    uint64_t* k_full = bars;
    uint64_t* k_empty = k_full + S;
    uint64_t* v_full = k_empty + S;
    uint64_t* v_empty = v_full + S;
    uint64_t* s_full = v_empty + S;
    // p_full[t & 1]: the four softmax warps wrote P(t).  Two barriers, because a warp may finish tile
    // t + 1 before a slower warp finishes tile t (it never gets two tiles ahead: S(t+2) is issued
    // after P.V(t), which waits for all four arrivals of tile t).
    uint64_t* p_full = s_full + 2;
    uint64_t* pv_done = p_full + 2;   // [t & 1] P.V(t) completed (waited by the S issuer, and by the
                                      // softmax before a rescale)
    uint64_t* drain = pv_done + 2;
    uint64_t* q_full = drain + 1;     // [2] Q tile of an item landed
    uint64_t* q_empty = q_full + 2;   // [2] the item's last S MMA completed: its Q buffer is free
    uint64_t* o_final = q_empty + 2;  // [2] the item's last P.V completed: O is final
    uint64_t* o_free = o_final + 2;   // [2] the epilogue has read O
    uint64_t* l_full = o_free + 2;
    uint64_t* xchg = l_full + LR;     // [tile parity][quarter] both halves of the rows wrote their maxima    // [LR] the item's row sums are in shared memory
    float* lsum = reinterpret_cast<float*>(sm + Sm::kL);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + Sm::kMisc);
    volatile int* abort = reinterpret_cast<volatile int*>(sm + Sm::kMisc + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_qt = (a.q_seq + kTcRows - 1) / kTcRows;
    const int n_items = a.q_heads * n_qt * a.batch;
    // Every role walks the same item sequence.  Key tiles of all items are numbered in one sequence
    // (t): stage t % S of the K/V ring, S and P buffer t & 1 (with its p_full / pv_done barrier).
    // Items that have key tiles are numbered z: Q and O buffer z & 1 (one q_full / q_empty /
    // o_final / o_free phase per item on that buffer's barrier) and row-sum slot z % LR.

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&q_full[i], 1);
            mbar_init(&q_empty[i], 1);
            mbar_init(&o_final[i], 1);
            mbar_init(&o_free[i], 4);
        }
        for (int i = 0; i < LR; ++i) mbar_init(&l_full[i], 8);  // both halves of every row
        for (int i = 0; i < 8; ++i) mbar_init(&xchg[i], 2);       // the two warps of a quarter
        mbar_init(&p_full[0], 8);
        mbar_init(&p_full[1], 8);
        mbar_init(&pv_done[0], 1);
        mbar_init(&pv_done[1], 1);
        mbar_init(drain, 2);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, kTcTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // Launched as a programmatic dependent of the kernel that wrote the bf16 operands (and the work
    // order): the set-up above touches only this CTA's shared memory and TMEM, and every global
    // access below comes after that grid has completed.  This kernel does not trigger its own
    // dependents early: they launch when it exits.
    asm volatile("griddepcontrol.wait;" ::: "memory");

    if (warp < 4) {
        reg_set<kTcRegsIssue>();
        if (warp == 0) {
            // ------------------------------------------------------------------ TMA producer
            if (lane == 0) {
                int t = 0, z = 0, issued = 0;  // issued: tiles whose copies are in flight or landed
                bool ok = true;
                uint64_t deadline = globaltimer_ns() + kWaitLimitNs;
                for (int w = 0; ok; ++w) {
                    const int idx = tc_walk(a, w, n_items);
                    if (idx < 0) break;
                    const TcItem it = tc_item(a, idx, n_qt);
                    if (it.n_kv == 0) continue;
                    deadline = globaltimer_ns() + kWaitLimitNs;
                    // Q of item z into buffer z & 1, once the last S MMA of item z - 2 has read it.
                    const int qb = z & 1;
                    if (z >= 2 &&
                        !tc_wait(&q_empty[qb], ((z >> 1) - 1) & 1, deadline, abort, a.err, KERR_TIMEOUT_EMPTY))
                        break;
                    mbar_arrive_expect_tx(&q_full[qb], Sm::kQBytes);
                    for (int c = 0; c < NCH; ++c)
                        tma_load_3d(sm + Sm::kQ + qb * Sm::kQBytes + c * Sm::kQChunkBytes, &tm_q, &q_full[qb], 64 * c,
                                    it.h, it.b * a.q_seq + it.r0);
                    ++z;
                    const int g = it.h / a.nrep, kv_row0 = it.b * a.kv_seq;
                    for (int j = 0; j < it.n_kv; ++j, ++t) {
                        const int s = t % S;
                        const uint32_t par = ((t / S) - 1) & 1;
                        if (t >= S && !tc_wait(&k_empty[s], par, deadline, abort, a.err, KERR_TIMEOUT_EMPTY)) {
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(&k_full[s], Sm::kKvBytes);
                        for (int c = 0; c < NCH; ++c)
                            tma_load_3d(sm + Sm::kK + s * Sm::kKvBytes + c * Sm::kKvChunkBytes, &tm_k, &k_full[s],
                                        64 * c, g, kv_row0 + j * kTcKeys);
                        if (t >= S && !tc_wait(&v_empty[s], par, deadline, abort, a.err, KERR_TIMEOUT_EMPTY)) {
                            ++issued;  // the K half of this stage is in flight
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(&v_full[s], Sm::kKvBytes);
                        for (int c = 0; c < NCH; ++c)
                            tma_load_3d(sm + Sm::kV + s * Sm::kKvBytes + c * Sm::kKvChunkBytes, &tm_v, &v_full[s],
                                        64 * c, g, kv_row0 + j * kTcKeys);
                        ++issued;
                    }
                }
                // Drain: the last copies issued into each buffer must land before the CTA exits.  No copy
                // is issued after these, so each barrier rests on the phase waited for here.
                const uint64_t dd = deadline + kWaitLimitNs / 2;
                for (int i = max(0, z - 2); i < z; ++i)
                    while (!mbar_try_wait(&q_full[i & 1], (i >> 1) & 1) && globaltimer_ns() < dd) {
                    }
                for (int j = max(0, issued - S); j < issued; ++j) {
                    const int s = j % S;
                    const uint32_t par = (j / S) & 1;
                    while (!mbar_try_wait(&k_full[s], par) && globaltimer_ns() < dd) {
                    }
                    while (!mbar_try_wait(&v_full[s], par) && globaltimer_ns() < dd) {
                    }
                }
            }
        } else if (warp == 1 || warp == kTcPvWarp) {
            // ------------------------------------------------------------------ MMA issuers
            // Two issuing threads on different SM sub-partitions: warp 1 issues S = Q.K^T, warp
            // kTcPvWarp issues O += P.V.  (An issuing thread shares its sub-partition with a softmax
            // warp, which slows its issue; two threads halve the MMAs each has to issue.)  MMAs of
            // different threads are not ordered, so S(t), which overwrites the S buffer that P(t-2) was
            // packed into, waits for pv_done(t-2).
            if (lane == 0) {
                constexpr uint32_t kIdS = idesc_bf16(kTcRows, kTcKeys, 0, 0);
                constexpr uint32_t kIdO = idesc_bf16(kTcRows, D, 0, 1);
                // Descriptors are built once and advanced by constant offsets: an issuing thread pays
                // the latency of every instruction between two MMAs.
                const uint64_t q_desc = smem_desc_sw128(smem_u32(sm + Sm::kQ), 16, 1024);
                const uint64_t k_desc = smem_desc_sw128(smem_u32(sm + Sm::kK), 16, 1024);
                const uint64_t v_desc = smem_desc_sw128(smem_u32(sm + Sm::kV), Sm::kKvChunkBytes, 1024);
                const bool is_s = warp == 1;
                bool ok = true;
                uint64_t deadline = globaltimer_ns() + kWaitLimitNs;
                int t = 0, z = 0;
                for (int w = 0; ok; ++w) {
                    const int idx = tc_walk(a, w, n_items);
                    if (idx < 0) break;
                    const int n_kv = tc_item(a, idx, n_qt).n_kv;
                    if (n_kv == 0) continue;
                    deadline = globaltimer_ns() + kWaitLimitNs;
                    const int qb = z & 1, ob = z & 1;
                    if (is_s) {
                        if (!tc_wait(&q_full[qb], (z >> 1) & 1, deadline, abort, a.err, KERR_TIMEOUT_FULL)) break;
                        const uint64_t qd = desc_advance(q_desc, qb * Sm::kQBytes);
                        for (int j = 0; j < n_kv; ++j, ++t) {
                            const int s = t % S, bf = t & 1;
                            if (!tc_wait(&k_full[s], (t / S) & 1, deadline, abort, a.err, KERR_TIMEOUT_FULL) ||
                                (t >= 2 && !tc_wait(&pv_done[bf], ((t >> 1) - 1) & 1, deadline, abort, a.err,
                                                    KERR_TIMEOUT_MMA))) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            const uint64_t kd = desc_advance(k_desc, s * Sm::kKvBytes);
                            const uint32_t d_tmem = tmem + Tm::kS + bf * kTcKeys;
#pragma unroll
                            for (int kk = 0; kk < D / 16; ++kk) {
                                const uint32_t qoff = (kk >> 2) * Sm::kQChunkBytes + (kk & 3) * 32;
                                const uint32_t koff = (kk >> 2) * Sm::kKvChunkBytes + (kk & 3) * 32;
                                umma_ss(d_tmem, desc_advance(qd, qoff), desc_advance(kd, koff), kIdS, kk > 0 ? 1u : 0u);
                            }
                            umma_commit(&s_full[bf]);
                            umma_commit(&k_empty[s]);
                            if (j == n_kv - 1) umma_commit(&q_empty[qb]);
                        }
                    } else {
                        for (int j = 0; j < n_kv; ++j, ++t) {
                            const int s = t % S, bf = t & 1;
                            // The first P.V of item z overwrites O buffer z & 1: item z - 2's epilogue must
                            // have read it.
                            if ((j == 0 && z >= 2 &&
                                 !tc_wait(&o_free[ob], ((z >> 1) - 1) & 1, deadline, abort, a.err, KERR_TIMEOUT_MMA)) ||
                                !tc_wait(&p_full[bf], (t >> 1) & 1, deadline, abort, a.err, KERR_TIMEOUT_MMA) ||
                                !tc_wait(&v_full[s], (t / S) & 1, deadline, abort, a.err, KERR_TIMEOUT_FULL)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            const uint32_t p_tmem = tmem + Tm::kS + bf * kTcKeys;  // P(t) packed in its S buffer
                            const uint32_t o_tmem = tmem + Tm::kO + ob * D;
                            const uint64_t vd = desc_advance(v_desc, s * Sm::kKvBytes);
                            umma_ts(o_tmem, p_tmem, vd, kIdO, j > 0 ? 1u : 0u);
#pragma unroll
                            for (int kk = 1; kk < kTcKeys / 16; ++kk)
                                umma_ts(o_tmem, p_tmem + kk * 8, desc_advance(vd, kk * 2048), kIdO, 1u);
                            umma_commit(&pv_done[bf]);
                            umma_commit(&v_empty[s]);
                            if (j == n_kv - 1) umma_commit(&o_final[ob]);
                        }
                    }
                    ++z;
                }
                // Drain: every MMA issued by either thread completes before TMEM is freed.
                umma_commit(drain);
                const uint64_t dd = deadline + kWaitLimitNs / 2;
                while (!mbar_try_wait(drain, 0) && globaltimer_ns() < dd) {
                }
            }
        }
    } else if (warp < 12) {
        reg_set<kTcRegsSoftmax>();
        // ------------------------------------------------------------------ softmax warpgroups
        // Two warpgroups split every S row: warps 4-7 take columns [0, 64), warps 8-11 columns
        // [64, 128) of the same TMEM lanes (warps w and w + 4 reach the same 32 lanes).  Per tile the
        // two threads of a row exchange their half-row maxima through shared memory (a named barrier
        // per warp pair, the buffer alternating by tile), so both use the same running max; each
        // exponentiates and packs its own 64 columns, rescales its half of O, and keeps its half of
        // the row sum, which the epilogue adds.  Two softmax warps per sub-partition instead of one
        // halve each thread's dependent chain.
        const int half = (warp - 4) >> 2;
        const int quarter = warp & 3;         // TMEM lanes [32*quarter, 32*quarter+32)
        const int row = quarter * 32 + lane;  // query row within the tile
        const uint32_t lane_off = uint32_t(quarter * 32) << 16;
        float* xmax = reinterpret_cast<float*>(sm + Sm::kX);  // [tile parity][half][128]
        constexpr int HK = kTcKeys / 2;                        // columns per half
        const float c2 = a.scale_log2;
        bool ok = true;
        int t = 0, z = 0;
        for (int w = 0; ok; ++w) {
            const int idx = tc_walk(a, w, n_items);
            if (idx < 0) break;
            const TcItem it = tc_item(a, idx, n_qt);
            if (it.n_kv == 0) continue;
            const uint64_t deadline = globaltimer_ns() + kWaitLimitNs;
            const int qr = it.r0 + row;  // query row within the sequence
            const int r0 = it.r0, kv_len = it.kv_len, n_kv = it.n_kv;
            const uint32_t o_tmem = tmem + Tm::kO + (z & 1) * D + lane_off;
            float m = -INFINITY, l = 0.f;
            for (int j = 0; j < n_kv; ++j, ++t) {
                const int bf = t & 1;
                const uint32_t s_tmem = tmem + Tm::kS + bf * kTcKeys + lane_off;
                const uint32_t s_half = s_tmem + half * HK;  // this half's S columns
                ok = __all_sync(0xffffffffu, ok && tc_wait(&s_full[bf], (t >> 1) & 1, deadline, abort, a.err,
                                                         KERR_TIMEOUT_MMA));
                if (!ok) break;
                tc_fence_after();
                const int k0 = j * kTcKeys;  // key position of column 0 (sequence-relative)
                const bool edge = (k0 + kTcKeys > kv_len) || (a.causal && k0 + kTcKeys - 1 > a.q_pos0 + r0);
                // Columns c < lim of this tile are visible to this row (key < kv_len, and key <= the
                // row's position under the causal mask).
                const int lim = min(kv_len - k0, a.causal ? a.q_pos0 + qr - k0 + 1 : kTcKeys);
                // The tile's row in registers (one read of TMEM; the softmax warpgroup's register
                // share holds it), then the row max over 8 independent chains of three-input max.
                uint32_t r[HK];
#pragma unroll
                for (int c = 0; c < HK; c += 32) tmem_ld32p(s_half + c, r + c);
                tmem_wait_ld();
                if (edge)
#pragma unroll
                    for (int c = 0; c < HK; ++c)
                        if (half * HK + c >= lim) r[c] = __float_as_uint(-INFINITY);
                float mx8[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) mx8[u] = fmaxf(__uint_as_float(r[u]), __uint_as_float(r[8 + u]));
#pragma unroll
                for (int c = 16; c < HK; c += 16)
#pragma unroll
                    for (int u = 0; u < 8; ++u)
                        mx8[u] = fmax3(mx8[u], __uint_as_float(r[c + u]), __uint_as_float(r[c + 8 + u]));
                const float mxh =
                    fmax3(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]));
                // The row max from both halves, exchanged through shared memory and an mbarrier per
                // warp pair (a bounded wait, so a partner that gave up cannot hang this warp).  The
                // buffer and barrier alternate by tile: this warp writes the slot of tile t + 2 only
                // after its partner's arrival for tile t + 1, which follows the partner's read of t.
                float* xm = xmax + (t & 1) * 2 * kTcRows;
                xm[half * kTcRows + row] = mxh;
                __syncwarp();
                uint64_t* xb = &xchg[(t & 1) * 4 + quarter];
                if (lane == 0) mbar_arrive(xb);
                ok = __all_sync(0xffffffffu, ok && tc_wait(xb, (t >> 1) & 1, deadline, abort, a.err, KERR_TIMEOUT_MMA));
                if (!ok) break;
                const float mx = fmaxf(mxh, xm[(1 - half) * kTcRows + row]);
                // The running max (log2 units) only moves when the tile max exceeds it by more than 8:
                // p = 2^(s*c2 - m) then stays <= 256 and O/l are rescaled rarely; the normalisation at
                // the end uses the same m, so the result is unchanged.
                const float mt = mx * c2;
                const float m_new = (m == -INFINITY || mt > m + 8.0f) ? mt : m;
                const float ms = m_new == -INFINITY ? 0.f : m_new;
                const float corr = (m == m_new || m_new == -INFINITY) ? 1.f : fast_exp2(m - m_new);
                m = m_new;
                // O holds P.V of tiles 0..j-1 of this item once pv_done(t-1) has completed.  It is
                // waited for only before a rescale (rare).  That wait is exact: the S issuer waited for
                // pv_done(t-3) before issuing S(t-1), which this warp has seen, and P.V(t+1) cannot
                // start before this warp's p_full(t+1).
                if (j >= 1 && __any_sync(0xffffffffu, corr != 1.f)) {
                    ok = __all_sync(0xffffffffu, ok && tc_wait(&pv_done[(t - 1) & 1], ((t - 1) >> 1) & 1, deadline,
                                                             abort, a.err, KERR_TIMEOUT_MMA));
                    if (!ok) break;
                    tc_fence_after();
                    uint32_t y[32];
#pragma unroll 1
                    for (int ch = half * (D / 64); ch < (half + 1) * (D / 64); ++ch) {  // this half's columns of O
                        tmem_ld32(o_tmem + ch * 32, y);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) y[i] = __float_as_uint(__uint_as_float(y[i]) * corr);
                        tmem_st32(o_tmem + ch * 32, y);
                    }
                    tmem_wait_st();
                }
                // p = 2^(s*c2 - ms) for key pairs, P packed as bf16 pairs (lower key in the low half:
                // the A-operand layout of a TMEM-sourced kind::f16 MMA) over the first kTcKeys/2
                // columns of the S buffer, which this thread has already read in full.  P of columns
                // [64h, 64h+64) lands in columns [32h, 32h+32).  Row sum over 4 pair accumulators.
                float2 rs4[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                                 make_float2(0.f, 0.f)};
                const float2 cc = make_float2(c2, c2), nm = make_float2(-ms, -ms);
                {
                    uint32_t pk[32];
#pragma unroll
                    for (int c = 0; c < 32; ++c) {
                        const int i = 2 * c;
                        float2 e = ffma2(make_float2(__uint_as_float(r[i]), __uint_as_float(r[i + 1])), cc, nm);
                        if ((kTcPolyPairs >> (c & 7)) & 1u) {
                            e = exp2_poly2(e);
                        } else {
                            e.x = fast_exp2(e.x);
                            e.y = fast_exp2(e.y);
                        }
                        pk[c] = pack_bf16(e.x, e.y);
                        rs4[c & 3] = fadd2(rs4[c & 3], e);
                    }
                    tmem_st32(s_tmem + half * 32, pk);  // P of columns [64h, 64h+64) into [32h, 32h+32)
                }
                const float2 rs2 = fadd2(fadd2(rs4[0], rs4[1]), fadd2(rs4[2], rs4[3]));
                l = l * corr + (rs2.x + rs2.y);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[bf]);
            }
            if (!ok) break;
            // The half-row sums go to the epilogue warps through shared memory.
            lsum[((z % LR) * 2 + half) * kTcRows + row] = l;
            __syncwarp();
            if (lane == 0) mbar_arrive(&l_full[z % LR]);
            ++z;
        }
        tc_fence_before();
    } else {
        reg_set<kTcRegsEpilogue>();
        // ------------------------------------------------------------------ epilogue warpgroup
        // Per item z: row sums from shared memory, O buffer z & 1 from TMEM once the last P.V has
        // completed, O / l to the output rows, then O buffer z & 1 is handed back to the MMA issuer.
        // A thread holds one row of O, so each warp passes 32 x 32 blocks through a padded staging
        // block and stores whole 128-byte row segments (8 lanes per row, 4 rows per instruction):
        // row-per-lane stores would touch 32 rows per instruction and crowd the shared-memory path
        // that the MMAs read their operands through.
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t lane_off = uint32_t(quarter * 32) << 16;
        float* stg = reinterpret_cast<float*>(sm + Sm::kE) + quarter * 32 * Sm::kStageRow;
        const int sub = lane >> 3, quad = lane & 7;  // transposed access: row 4k + sub, columns 4*quad..
        bool ok = true;
        uint32_t x[32];
        int z = 0;
        for (int w = 0; ok; ++w) {
            const int idx = tc_walk(a, w, n_items);
            if (idx < 0) break;
            const TcItem it = tc_item(a, idx, n_qt);
            const int row0 = it.r0 + quarter * 32;  // first sequence row of this warp's 32 rows
            float* obase = a.out + ((static_cast<size_t>(it.b) * a.q_seq + row0) * a.q_heads + it.h) * D;
            const size_t ostride = static_cast<size_t>(a.q_heads) * D;  // floats between rows
            if (it.n_kv == 0) {  // padded query rows only: zeros, D/4 lanes per row
                constexpr int F4 = D / 4, RPI = 32 / F4;
#pragma unroll
                for (int rr = lane / F4; rr < 32; rr += RPI)
                    if (row0 + rr < a.q_seq)
                        *reinterpret_cast<float4*>(obase + rr * ostride + 4 * (lane % F4)) =
                            make_float4(0.f, 0.f, 0.f, 0.f);
                continue;
            }
            const uint64_t deadline = globaltimer_ns() + kWaitLimitNs;
            const int ob = z & 1;
            ok = __all_sync(0xffffffffu, tc_wait(&l_full[z % LR], (z / LR) & 1, deadline, abort, a.err,
                                                 KERR_TIMEOUT_MMA));
            if (!ok) break;
            // Padded rows (past the valid ones) are written as zeros.
            const float inv = it.r0 + row < it.nq_valid
                                  ? 1.0f / (lsum[(z % LR) * 2 * kTcRows + row] + lsum[((z % LR) * 2 + 1) * kTcRows + row])
                                  : 0.f;
            ok = __all_sync(0xffffffffu, tc_wait(&o_final[ob], (z >> 1) & 1, deadline, abort, a.err,
                                                 KERR_TIMEOUT_MMA));
            if (!ok) break;
            tc_fence_after();
#pragma unroll 1
            for (int ch = 0; ch < D / 32; ++ch) {
                tmem_ld32(tmem + Tm::kO + ob * D + ch * 32 + lane_off, x);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; i += 4)
                    *reinterpret_cast<float4*>(stg + lane * Sm::kStageRow + i) =
                        make_float4(__uint_as_float(x[i]) * inv, __uint_as_float(x[i + 1]) * inv,
                                    __uint_as_float(x[i + 2]) * inv, __uint_as_float(x[i + 3]) * inv);
                __syncwarp();
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const int rr = 4 * k + sub;
                    if (row0 + rr < a.q_seq)
                        *reinterpret_cast<float4*>(obase + rr * ostride + ch * 32 + 4 * quad) =
                            *reinterpret_cast<const float4*>(stg + rr * Sm::kStageRow + 4 * quad);
                }
                __syncwarp();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&o_free[ob]);
            ++z;
        }
        tc_fence_before();
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTcTmemCols);
    }
}

}  // namespace lg
