// flash_tc.cuh - bf16 tensor-core attention (tcgen05 + TMEM + TMA) for causal prefill and BERT.
//
// Same semantics as flash_simt.cuh (prefill = the reference's one-token-at-a-time loop,
// fast/ligguf_fast_qk.cpp:340-356; BERT = fast/vdb.cpp:189-212 per sequence), with q, k, v rounded
// to bf16 and every product accumulated in fp32 by the tensor cores.
//
// CTA = 128 query rows of one q head (of one batch entry), 192 threads, two CTAs per SM (96 KB of
// shared memory and 256 TMEM columns each) so that one CTA's MMAs run while the other's softmax
// warps work:
//   warp 0      TMA producer: Q tile once, then K and V tiles (64 keys each) into 2-stage rings
//   warp 1      allocates 256 TMEM columns; lane 0 issues every tcgen05.mma and commit
//   warps 2..5  softmax: thread = query row = TMEM lane; reads S from TMEM, online softmax with
//               exp2, writes P as bf16 pairs back into the same TMEM columns, rescales O in TMEM
//               when the running max moves; final O / l to global memory.
// TMEM: S double buffer at columns [0,64) and [64,128) (P of a tile overwrites the first 32 columns
// of its S buffer), O at [128, 128+D).  MMA order S0, S1, PV0, S2, PV1, ...: S = Q.K^T with both
// operands in shared memory (K-major, SWIZZLE_128B); O += P.V with P read from TMEM and V from
// shared memory (MN-major, SWIZZLE_128B).  MMAs of one CTA execute in issue order, so PV(j) has read
// P(j) before S(j+2) overwrites that buffer.  Every wait is bounded; on a timeout the kernel records
// an error, drains its own copies and MMAs, frees TMEM and returns.
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
};

__global__ void to_bf16_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst, size_t n) {
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
        dst[i] = __float2bfloat16_rn(src[i]);
}

// BERT operands to bf16 in one pass, valid rows only: rows r < lens[b] of q, k and v are converted;
// padded rows of v are written as zeros (P.V multiplies them by P = 0, so they must be finite), while
// padded rows of q and k are left as they are (their scores are masked or their outputs discarded).
// Block = kBertConvRows rows of one batch entry; 8 values per thread step (two 16-byte loads, one
// 16-byte store).  Needs E % 8 == 0 and 16-byte aligned bases.
constexpr int kBertConvRows = 8;
__global__ void __launch_bounds__(256) bert_to_bf16_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                                           const float* __restrict__ v, const int* __restrict__ lens,
                                                           int max_len, int E, __nv_bfloat16* __restrict__ bq,
                                                           __nv_bfloat16* __restrict__ bk, __nv_bfloat16* __restrict__ bv) {
    const int b = blockIdx.y;
    const int r0 = blockIdx.x * kBertConvRows;
    const int len = min(lens[b], max_len);
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
            if (t == 2) *reinterpret_cast<uint4*>(dst + off) = make_uint4(0u, 0u, 0u, 0u);
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

constexpr int kTcRows = 128;  // query rows per tile (UMMA M)
constexpr int kTcKeys = 64;   // keys per tile (UMMA N of S, K of P.V)
constexpr int kTcThreads = 192;
constexpr uint32_t kTcTmemCols = 256;
constexpr uint32_t kTcTmemO = 128;  // first TMEM column of O

template <int D>
struct TcSmem {
    static constexpr int kChunks = D / 64;               // 128-byte column chunks of a row
    static constexpr int kQBytes = kTcRows * D * 2;      // the Q tile: 128 rows of bf16
    static constexpr int kQChunkBytes = kTcRows * 128;   // one 128-byte-wide chunk of Q
    static constexpr int kKvBytes = kTcKeys * D * 2;     // a K or V tile: 64 rows of bf16
    static constexpr int kKvChunkBytes = kTcKeys * 128;  // one 128-byte-wide chunk of a K/V tile
    // D = 64 takes 4 stages: besides the deeper ring, 80 KB keeps a third CTA (whose TMEM allocation
    // would have to wait for one of the two resident CTAs to finish) off the SM.
    static constexpr int kStages = D == 128 ? 2 : 4;
    static constexpr size_t kQ = 0;
    static constexpr size_t kK = kQ + kQBytes;
    static constexpr size_t kV = kK + size_t(kStages) * kKvBytes;
    static constexpr size_t kBar = kV + size_t(kStages) * kKvBytes;
    // q_full, k_full[S], k_empty[S], v_full[S], v_empty[S], s_full[2], s_free[2], p_full, o_done, drain
    static constexpr int kNumBars = 1 + 4 * kStages + 2 + 2 + 1 + 1 + 1;
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
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

template <int D>
__global__ void __launch_bounds__(kTcThreads, 2)
    flash_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const TcArgs a) {
    using Sm = TcSmem<D>;
    constexpr int S = Sm::kStages;
    constexpr int NCH = Sm::kChunks;
    extern __shared__ uint8_t tc_smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Sm::kBar);
    uint64_t* q_full = bars;
    uint64_t* k_full = bars + 1;
    uint64_t* k_empty = k_full + S;
    uint64_t* v_full = k_empty + S;
    uint64_t* v_empty = v_full + S;
    uint64_t* s_full = v_empty + S;
    uint64_t* s_free = s_full + 2;
    uint64_t* p_full = s_free + 2;
    uint64_t* o_done = p_full + 1;
    uint64_t* drain = o_done + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + Sm::kMisc);
    volatile int* abort = reinterpret_cast<volatile int*>(sm + Sm::kMisc + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_qt = (a.q_seq + kTcRows - 1) / kTcRows;
    // Blocks start in linear order (x fastest): x = head, y = query tile from the last (longest under
    // the causal mask) to the first, so every wave takes the heaviest remaining tiles of all heads.
    const int h = blockIdx.x, b = blockIdx.z;
    const int qt = n_qt - 1 - static_cast<int>(blockIdx.y);
    const int g = h / a.nrep;
    const int r0 = qt * kTcRows;
    const int nq_valid = a.lens ? min(a.lens[b], a.q_seq) : a.q_seq;
    const int kv_len = a.lens ? min(a.lens[b], a.kv_seq) : a.kv_seq;
    const uint64_t deadline = globaltimer_ns() + kWaitLimitNs;

    if (r0 >= nq_valid) {  // padded query rows only: zeros (uniform for the CTA)
        for (int i = threadIdx.x; i < kTcRows * D; i += kTcThreads) {
            const int r = r0 + i / D;
            if (r < a.q_seq)
                a.out[((static_cast<size_t>(b) * a.q_seq + r) * a.q_heads + h) * D + (i % D)] = 0.f;
        }
        return;
    }
    int kv_eff = kv_len;
    if (a.causal) kv_eff = min(kv_eff, a.q_pos0 + min(r0 + kTcRows, nq_valid));
    const int n_kv = (kv_eff + kTcKeys - 1) / kTcKeys;
    const int q_row0 = b * a.q_seq + r0;
    const int kv_row0 = b * a.kv_seq;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < S; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], 4);
        }
        mbar_init(p_full, 4);
        mbar_init(o_done, 1);
        mbar_init(drain, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, kTcTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tmem_s0 = tmem, tmem_o = tmem + kTcTmemO;

    if (warp == 0) {
        // ------------------------------------------------------------------ TMA producer
        if (lane == 0) {
            int issued = 0;
            mbar_arrive_expect_tx(q_full, Sm::kQBytes);
            for (int c = 0; c < NCH; ++c)
                tma_load_3d(sm + Sm::kQ + c * Sm::kQChunkBytes, &tm_q, q_full, 64 * c, h, q_row0);
            for (int j = 0; j < n_kv; ++j) {
                const int s = j % S;
                const uint32_t par = ((j / S) - 1) & 1;
                if (j >= S && !tc_wait(&k_empty[s], par, deadline, abort, a.err, KERR_TIMEOUT_EMPTY)) break;
                mbar_arrive_expect_tx(&k_full[s], Sm::kKvBytes);
                for (int c = 0; c < NCH; ++c)
                    tma_load_3d(sm + Sm::kK + s * Sm::kKvBytes + c * Sm::kKvChunkBytes, &tm_k, &k_full[s], 64 * c,
                                g, kv_row0 + j * kTcKeys);
                if (j >= S && !tc_wait(&v_empty[s], par, deadline, abort, a.err, KERR_TIMEOUT_EMPTY)) {
                    ++issued;  // the K half of this stage is in flight
                    break;
                }
                mbar_arrive_expect_tx(&v_full[s], Sm::kKvBytes);
                for (int c = 0; c < NCH; ++c)
                    tma_load_3d(sm + Sm::kV + s * Sm::kKvBytes + c * Sm::kKvChunkBytes, &tm_v, &v_full[s], 64 * c,
                                g, kv_row0 + j * kTcKeys);
                ++issued;
            }
            // Drain: the last copies issued into each stage must land before the CTA exits.
            const uint64_t dd = deadline + kWaitLimitNs / 2;
            while (!mbar_try_wait(q_full, 0) && globaltimer_ns() < dd) {
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
    } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t kIdS = idesc_bf16(kTcRows, kTcKeys, 0, 0);
            constexpr uint32_t kIdO = idesc_bf16(kTcRows, D, 0, 1);
            // Descriptors are built once and advanced by constant offsets: a single issuing thread
            // pays the latency of every instruction between two MMAs.
            const uint64_t q_desc = smem_desc_sw128(smem_u32(sm + Sm::kQ), 16, 1024);
            const uint64_t k_desc = smem_desc_sw128(smem_u32(sm + Sm::kK), 16, 1024);
            const uint64_t v_desc = smem_desc_sw128(smem_u32(sm + Sm::kV), Sm::kKvChunkBytes, 1024);
            bool ok = tc_wait(q_full, 0, deadline, abort, a.err, KERR_TIMEOUT_FULL);
            auto issue_pv = [&](int i) -> bool {
                const int s = i % S;
                if (!tc_wait(p_full, i & 1, deadline, abort, a.err, KERR_TIMEOUT_MMA)) return false;
                if (!tc_wait(&v_full[s], (i / S) & 1, deadline, abort, a.err, KERR_TIMEOUT_FULL)) return false;
                tc_fence_after();
                const uint32_t p_tmem = tmem_s0 + (i & 1) * kTcKeys;  // P(i) packed in its S buffer
                const uint64_t vd = desc_advance(v_desc, s * Sm::kKvBytes);
                umma_ts(tmem_o, p_tmem, vd, kIdO, i > 0 ? 1u : 0u);
#pragma unroll
                for (int kk = 1; kk < kTcKeys / 16; ++kk)
                    umma_ts(tmem_o, p_tmem + kk * 8, desc_advance(vd, kk * 2048), kIdO, 1u);
                umma_commit(o_done);
                umma_commit(&v_empty[s]);
                return true;
            };
            for (int j = 0; ok && j < n_kv; ++j) {
                const int s = j % S, bf = j & 1;
                if (!tc_wait(&k_full[s], (j / S) & 1, deadline, abort, a.err, KERR_TIMEOUT_FULL)) break;
                if (j >= 2 && !tc_wait(&s_free[bf], ((j >> 1) - 1) & 1, deadline, abort, a.err, KERR_TIMEOUT_MMA))
                    break;
                tc_fence_after();
                const uint64_t kd = desc_advance(k_desc, s * Sm::kKvBytes);
                const uint32_t d_tmem = tmem_s0 + bf * kTcKeys;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t qoff = (kk >> 2) * Sm::kQChunkBytes + (kk & 3) * 32;
                    const uint32_t koff = (kk >> 2) * Sm::kKvChunkBytes + (kk & 3) * 32;
                    umma_ss(d_tmem, desc_advance(q_desc, qoff), desc_advance(kd, koff), kIdS, kk > 0 ? 1u : 0u);
                }
                umma_commit(&s_full[bf]);
                umma_commit(&k_empty[s]);
                if (j >= 1 && !issue_pv(j - 1)) {
                    ok = false;
                    break;
                }
            }
            if (ok && !*abort) issue_pv(n_kv - 1);
            // Drain: every MMA issued above completes before TMEM is freed.
            umma_commit(drain);
            const uint64_t dd = deadline + kWaitLimitNs / 2;
            while (!mbar_try_wait(drain, 0) && globaltimer_ns() < dd) {
            }
        }
    } else {
        // ------------------------------------------------------------------ softmax warpgroup
        const int quarter = warp & 3;                  // TMEM lanes [32*quarter, 32*quarter+32)
        const int row = quarter * 32 + lane;           // query row within the tile
        const int qr = r0 + row;                       // query row within the sequence
        const bool row_valid = qr < nq_valid;
        const uint32_t lane_off = uint32_t(quarter * 32) << 16;
        const float c2 = a.scale_log2;
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        uint32_t x[32];
        for (int j = 0; j < n_kv; ++j) {
            const int bf = j & 1;
            ok = __all_sync(0xffffffffu, ok && tc_wait(&s_full[bf], (j >> 1) & 1, deadline, abort, a.err,
                                                     KERR_TIMEOUT_MMA));
            if (!ok) break;
            tc_fence_after();
            uint32_t raw[kTcKeys];
#pragma unroll
            for (int ch = 0; ch < kTcKeys / 32; ++ch)
                tmem_ld32p(tmem_s0 + bf * kTcKeys + ch * 32 + lane_off, raw + ch * 32);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_free[bf]);
            float sv[kTcKeys];
#pragma unroll
            for (int c = 0; c < kTcKeys; ++c) sv[c] = __uint_as_float(raw[c]);

            const int k0 = j * kTcKeys;  // key position of column 0 (sequence-relative)
            const bool edge = (k0 + kTcKeys > kv_len) || (a.causal && k0 + kTcKeys - 1 > a.q_pos0 + r0);
            if (edge) {
                const int lim_c = kv_len - k0;
                const int lim_r = a.causal ? a.q_pos0 + qr - k0 : kTcKeys;
#pragma unroll
                for (int c = 0; c < kTcKeys; ++c) sv[c] = (c < lim_c && c <= lim_r) ? sv[c] : -INFINITY;
            }
            // Row max with 8 independent chains of three-input max.
            float mx8[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) mx8[u] = sv[u];
#pragma unroll
            for (int c = 8; c < kTcKeys; c += 16)
#pragma unroll
                for (int u = 0; u < 8; ++u) mx8[u] = fmax3(mx8[u], sv[c + u], sv[c + 8 + u]);
            const float mx = fmax3(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]));
            // The running max (log2 units) only moves when the tile max exceeds it by more than 8:
            // p = 2^(s*c2 - m) then stays <= 256 and O/l are rescaled rarely; the normalisation at
            // the end uses the same m, so the result is unchanged.
            const float mt = mx * c2;
            const float m_new = (m == -INFINITY || mt > m + 8.0f) ? mt : m;
            const float ms = m_new == -INFINITY ? 0.f : m_new;
            const float corr = (m == m_new || m_new == -INFINITY) ? 1.f : fast_exp2(m - m_new);
            // p = 2^(s*c2 - ms) for key pairs, P packed as bf16 pairs (lower key in the low half: the
            // A-operand layout of a TMEM-sourced kind::f16 MMA), row sum over 4 pair accumulators.
            float2 rs4[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
            const float2 cc = make_float2(c2, c2), nm = make_float2(-ms, -ms);
#pragma unroll
            for (int c = 0; c < kTcKeys / 2; ++c) {
                float2 t = ffma2(make_float2(sv[2 * c], sv[2 * c + 1]), cc, nm);
                t.x = fast_exp2(t.x);
                t.y = fast_exp2(t.y);
                x[c] = pack_bf16(t.x, t.y);
                rs4[c & 3] = fadd2(rs4[c & 3], t);
            }
            const float2 rs2 = fadd2(fadd2(rs4[0], rs4[1]), fadd2(rs4[2], rs4[3]));
            l = l * corr + (rs2.x + rs2.y);
            m = m_new;
            // O holds PV(0..j-1).  Wait for PV(j-1) on every tile, also when O needs no rescale: a
            // parity wait is only exact while the waiter never falls two phases behind the barrier
            // or gets two ahead of it (skipping waits would let the epilogue's wait return before
            // the last P.V landed).  O is rescaled only when the max moved by more than 2^8 (rare).
            if (j >= 1) {
                ok = __all_sync(0xffffffffu, ok && tc_wait(o_done, (j - 1) & 1, deadline, abort, a.err,
                                                         KERR_TIMEOUT_MMA));
                if (!ok) break;
                tc_fence_after();
            }
            if (j >= 1 && __any_sync(0xffffffffu, corr != 1.f)) {
                uint32_t y[32];
#pragma unroll 1
                for (int ch = 0; ch < D / 32; ++ch) {
                    tmem_ld32(tmem_o + ch * 32 + lane_off, y);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) y[i] = __float_as_uint(__uint_as_float(y[i]) * corr);
                    tmem_st32(tmem_o + ch * 32 + lane_off, y);
                }
                tmem_wait_st();
            }
            // P row -> TMEM over the S buffer just read.
            tmem_st32(tmem_s0 + bf * kTcKeys + lane_off, x);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
        }
        if (ok && !*abort) {
            ok = __all_sync(0xffffffffu, tc_wait(o_done, (n_kv - 1) & 1, deadline, abort, a.err, KERR_TIMEOUT_MMA));
            if (ok) {
                tc_fence_after();
                const float inv = 1.0f / l;
                float* orow = a.out + ((static_cast<size_t>(b) * a.q_seq + qr) * a.q_heads + h) * D;
#pragma unroll
                for (int ch = 0; ch < D / 32; ++ch) {
                    tmem_ld32(tmem_o + ch * 32 + lane_off, x);
                    tmem_wait_ld();
                    if (row_valid) {
#pragma unroll
                        for (int i = 0; i < 32; i += 4)
                            *reinterpret_cast<float4*>(orow + ch * 32 + i) =
                                make_float4(__uint_as_float(x[i]) * inv, __uint_as_float(x[i + 1]) * inv,
                                            __uint_as_float(x[i + 2]) * inv, __uint_as_float(x[i + 3]) * inv);
                    } else if (qr < a.q_seq) {
#pragma unroll
                        for (int i = 0; i < 32; i += 4)
                            *reinterpret_cast<float4*>(orow + ch * 32 + i) = make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                }
            }
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
