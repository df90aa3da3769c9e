// qmatvec.cuh - the QKV projection of the FAST forward pass on the GPU: quantized matrix-vector (and
// few-token matrix) products over GGUF weight blocks held in HBM, with the reference's activation
// quantization.
//
// Replaces (fast/lil_math.cpp):
//   quantize_q8_K (:352-385) and quantize_q8_0 (:329-350), the activation quantizers;
//   matmul3 (:827-899), matmul2 and matmul (:757-825): out[r] = dot(row r of W, x) per weight type,
//   through the per-type dots dot_f32 .. dot_q8_K_q6_K (:389-778; AVX2 versions fast/arch_avx2.h).
// The weight types are the reference's (gguf_type numbers, fast/lil_gguf.h:26-44): F32, F16, Q8_0,
// Q1_0, Q1_G against the Q8_0-quantized activation, Q2_K .. Q6_K against the Q8_K-quantized one.
// A launch takes up to T tokens (x rows): the result equals T separate matmul3 calls, which is what
// the engine's token-by-token prompt loop does (feed_text, fast/ligguf_fast_qk.cpp:340-356).
//
// Arithmetic: the quantized activation is bit-identical to the reference's (the integer values,
// block scales and 16-element sums).  Every weight block is split into 32-element units; a unit's
// integer dot product (dp4a over eight 4-byte words) and its per-16 or per-32 scale terms are exact
// integers, as in the reference; only the order in which the fp32 unit terms are summed differs.
//
// Kernel layout (one CTA per SM, persistent over a contiguous share of row tiles): warp kQmvWarps
// streams whole row tiles (rows are contiguous in HBM) with 1-D bulk copies into a ring of shared
// memory stages; the consumer warps quantize the x rows into shared memory once (every CTA quantizes
// them all: a few KB per token, read from L2), then each warp takes rows of the tile and each lane a
// 32-element unit of the row at a time, unpacking the unit's weights once for all T tokens.  The
// weights do not depend on the previous kernel in the stream, so the producer starts streaming
// before the previous grid completes (programmatic dependent launch); the consumers wait for it
// before reading x.
#pragma once

#include "common.cuh"

namespace lg {

// GGUF type numbers (fast/lil_gguf.h:26-44).
enum : int { QT_F32 = 0, QT_F16 = 1, QT_Q8_0 = 8, QT_Q2_K = 10, QT_Q3_K = 11, QT_Q4_K = 12, QT_Q5_K = 13,
             QT_Q6_K = 14, QT_Q1_0 = 40, QT_Q1_G = 41,
             QT_Q8_0_G32 = 108 };  // (internal) Q8_0 repacked at upload, see WUnit<QT_Q8_0_G32>

// Bytes and elements of one block of a type (fast/lil_gguf.h:64-119); 0 for an unknown type.
__host__ __device__ constexpr int qt_block_bytes(int t) {
    return t == QT_F32 ? 4 : t == QT_F16 ? 2 : t == QT_Q8_0 ? 34 : t == QT_Q1_0 ? 6 : t == QT_Q1_G ? 18
         : t == QT_Q2_K ? 84 : t == QT_Q3_K ? 110 : t == QT_Q4_K ? 144 : t == QT_Q5_K ? 176
         : t == QT_Q6_K ? 210 : 0;
}
__host__ __device__ constexpr int qt_block_elems(int t) {
    return t == QT_F32 || t == QT_F16 ? 1 : t == QT_Q8_0 || t == QT_Q1_0 ? 32 : t == QT_Q1_G ? 128
         : qt_block_bytes(t) ? 256 : 0;
}
// Which activation form a type's dot reads (matmul3 quantizes to Q8_0 for Q8_0/Q1_0/Q1_G,
// fast/lil_math.cpp:830-834; the engine passes the Q8_K form for the K-quants, :39-40).
__host__ __device__ constexpr bool qt_uses_q8k(int t) { return t >= QT_Q2_K && t <= QT_Q6_K; }
__host__ __device__ constexpr bool qt_uses_q80(int t) {
    return t == QT_Q8_0 || t == QT_Q8_0_G32 || t == QT_Q1_0 || t == QT_Q1_G;
}
__host__ __device__ constexpr bool qt_uses_f32(int t) { return t == QT_F32 || t == QT_F16; }

// 7 consumer warps + 1 producer warp, two CTAs per SM (14 consumer warps per SM; the consumers are
// latency-bound, so resident warps are what sets the pace).  The ring depth (2..4 stages of up to
// 32 KB) is chosen per launch so that two CTAs fit an SM's shared memory.
constexpr int kQmvWarps = 7;                        // consumer warps
constexpr int kQmvThreads = (kQmvWarps + 1) * 32;   // + the producer warp
constexpr int kQmvMaxStages = 4;
constexpr int kQmvStageMax = 32 * 1024;              // bytes of one ring stage (a tile of rows)
constexpr int kQmvMaxN = 16384;                      // input width limit (activation in shared memory)
constexpr int kQmvMaxMats = 3;
constexpr int kQmvMaxTokens = 8;                     // x rows per launch

struct QmvMat {
    const uint8_t* w;  // rows of `rb` bytes, 16-byte aligned base, allocation padded to 16 bytes
    float* out;        // out[t * out_stride + r]
    long long out_stride;
    int type, rows, rb, tile_rows, tile0, ntiles;
};

// Shared-memory layout of one token's quantized activation (byte offsets within the token's region;
// token t's region starts at t * tok_bytes).
struct QmvAct {
    int off_qk, off_dk, off_bs;  // q8_K: int8 [n], float [n/256], int [n/16]
    int off_q0, off_d0;          // q8_0: int8 [n], float [n/32] (the fp16-rounded scale)
    int off_xf;                  // fp32 x [n]
    int tok_bytes;               // bytes of one token's region (16-byte multiple)
    int bytes;                   // all tokens, a multiple of 1024 (the ring starts after it)
};

// Reduce mode (the SARA attn_output partial, cpp/ligguf_distrib.cpp:749-750): instead of out[r], row
// r's value goes to every rank's reduce buffer [2][nranks][rows] as one 64-bit word (epoch << 32) |
// fp32 bits, at [epoch & 1][rank][r]; the epoch is state[0] + 1 (state[0] is advanced by the reduce
// wait kernel).  One token, one matrix.
struct QmvRed {
    unsigned long long* const* peers;  // [nranks] reduce buffer bases (null: plain outputs)
    const int* state;
    int nranks, rank;
};

struct QmvArgs {
    QmvRed red;
    QmvMat m[kQmvMaxMats];
    int nmat;
    const uint8_t* act_g;  // the tokens' activation forms (layout `act`), written by qmv_act_kernel, or
    const float* x;        // null: one token's x, quantized by this kernel (T = 1)
    int n_tok;             // tokens in this launch (<= the kernel's T)
    int n;
    int need_k, need_0, need_f;
    int ntiles;      // over all matrices
    int stages;      // ring depth, 2..kQmvMaxStages
    QmvAct act;
    int* err;
};

// ------------------------------------------------------------------------------ quantizers
// Round half away from zero to int, as nearest_int (fast/lil_math.cpp:347-350): (int)(f +- 0.5f),
// each operation rounded to fp32.
__device__ __forceinline__ int nearest_int_ref(float f) {
    return f < 0.f ? __float2int_rz(__fsub_rn(f, 0.5f)) : __float2int_rz(__fadd_rn(f, 0.5f));
}

// One 256-element block of quantize_q8_K (fast/lil_math.cpp:352-385) by one warp; lane l holds
// elements [8l, 8l+8).  max = the first element of largest magnitude; iscale = -127/max (an IEEE
// division); q = min(127, nearest_int(iscale*x)); d = max * (-1/127), the form the reference's
// -Ofast build computes 1/iscale in (checked against the compiled reference).  Writes q, d and the
// 16 sums of 16 to the given destinations (q and sums indexed within the block).
__device__ __forceinline__ void q8k_block_vals(const float (&v)[8], int8_t* q, float* d, int* bs_int, int16_t* bs_i16,
                                               int lane) {
    float amax = 0.f, mx = 0.f;
    int idx = 1 << 30;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float ax = fabsf(v[i]);
        if (ax > amax) {
            amax = ax;
            mx = v[i];
            idx = 8 * lane + i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {  // larger magnitude wins; the lower index on a tie
        const float oa = __shfl_xor_sync(0xffffffffu, amax, o);
        const float om = __shfl_xor_sync(0xffffffffu, mx, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (oa > amax || (oa == amax && oi < idx)) {
            amax = oa;
            mx = om;
            idx = oi;
        }
    }
    int qi[8];
    int s = 0;
    if (amax == 0.f) {
#pragma unroll
        for (int i = 0; i < 8; ++i) qi[i] = 0;
    } else {
        const float iscale = __fdiv_rn(-127.0f, mx);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            qi[i] = min(127, nearest_int_ref(__fmul_rn(iscale, v[i])));
            s += qi[i];
        }
    }
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        w0 |= (uint32_t(qi[i]) & 0xFFu) << (8 * i);
        w1 |= (uint32_t(qi[i + 4]) & 0xFFu) << (8 * i);
    }
    reinterpret_cast<uint2*>(q)[lane] = make_uint2(w0, w1);
    const int s16 = s + __shfl_xor_sync(0xffffffffu, s, 1);  // lanes 2g, 2g+1 hold group g
    if ((lane & 1) == 0) {
        if (bs_int) bs_int[lane >> 1] = s16;
        if (bs_i16) bs_i16[lane >> 1] = static_cast<int16_t>(s16);
    }
    if (lane == 0) *d = amax == 0.f ? 0.f : __fmul_rn(mx, -1.0f / 127.0f);
}
__device__ __forceinline__ void q8k_block_warp(const float* __restrict__ x, int8_t* q, float* d, int* bs_int,
                                               int16_t* bs_i16, int lane) {
    const float4 a = reinterpret_cast<const float4*>(x)[2 * lane];
    const float4 b = reinterpret_cast<const float4*>(x)[2 * lane + 1];
    const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    q8k_block_vals(v, q, d, bs_int, bs_i16, lane);
}

// One 32-element block of quantize_q8_0 (fast/lil_math.cpp:329-350) by one warp, lane = element:
// q = roundf(x * id), the block keeps d as fp16.  The reference's -Ofast build computes d = amax/127
// as amax * (1/127) and id = 1/d as 127/amax (both checked against the compiled reference on
// millions of blocks); so does this.  Returns q to the lane; lane 0 gets the fp16 bits of d.
__device__ __forceinline__ int q80_block_warp(float xv, uint16_t* d_bits, int lane) {
    float amax = fabsf(xv);
    amax = warp_max(amax);
    const float d = __fmul_rn(amax, 1.0f / 127.0f);
    const float id = d != 0.f ? __fdiv_rn(127.0f, amax) : 0.f;
    if (lane == 0) *d_bits = __half_as_ushort(__float2half_rn(d));
    return static_cast<int>(roundf(__fmul_rn(xv, id)));
}

// The same block by one thread: the 32 values in registers, amax over them (the order of a max does
// not matter), then the same d, 1/d and rounding; writes the 32 q values and d (as its fp32 value).
__device__ __forceinline__ void q80_block_lane(const float* __restrict__ x, int8_t* q, float* d_out) {
    float v[32];
    const float4* x4 = reinterpret_cast<const float4*>(x);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 f = x4[i];
        v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const float d = __fmul_rn(amax, 1.0f / 127.0f);
    const float id = d != 0.f ? __fdiv_rn(127.0f, amax) : 0.f;
    uint32_t* qw = reinterpret_cast<uint32_t*>(q);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        uint32_t w = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j)
            w |= uint32_t(uint8_t(static_cast<int8_t>(static_cast<int>(roundf(__fmul_rn(v[4 * i + j], id)))))) << (8 * j);
        qw[i] = w;
    }
    *d_out = __half2float(__float2half_rn(d));
}

// ------------------------------------------------------------------------------ unit dots
// One token's activation forms in shared memory.
struct QmvActView {
    const int8_t* qk;
    const float* dk;
    const int* bs;
    const int8_t* q0;
    const float* d0;
    const float* xf;
};

__device__ __forceinline__ QmvActView act_view(const uint8_t* base, const QmvAct& a, int t) {
    const uint8_t* b = base + size_t(t) * a.tok_bytes;
    QmvActView v;
    v.qk = reinterpret_cast<const int8_t*>(b + a.off_qk);
    v.dk = reinterpret_cast<const float*>(b + a.off_dk);
    v.bs = reinterpret_cast<const int*>(b + a.off_bs);
    v.q0 = reinterpret_cast<const int8_t*>(b + a.off_q0);
    v.d0 = reinterpret_cast<const float*>(b + a.off_d0);
    v.xf = reinterpret_cast<const float*>(b + a.off_xf);
    return v;
}

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t lds16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }
// Eight 4-byte words starting at a 2-byte aligned address (nine aligned loads and funnel shifts).
__device__ __forceinline__ void load8_a2(const uint8_t* p, uint32_t (&w)[8]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t* b = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
    const uint32_t sh = uint32_t(a & 3) * 8;
    uint32_t r[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) r[i] = b[i];
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = __funnelshift_r(r[i], r[i + 1], sh);
}
// Same from a 16-byte aligned address: two 16-byte loads.
__device__ __forceinline__ void load8_a16(const uint8_t* p, uint32_t (&w)[8]) {
    const uint4 lo = lds128(p), hi = lds128(p + 16);
    w[0] = lo.x; w[1] = lo.y; w[2] = lo.z; w[3] = lo.w;
    w[4] = hi.x; w[5] = hi.y; w[6] = hi.z; w[7] = hi.w;
}
__device__ __forceinline__ void load8_a4(const uint8_t* p, uint32_t (&w)[8]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = reinterpret_cast<const uint32_t*>(p)[i];
}
// Activation words of unit u (32 int8 values).
__device__ __forceinline__ void act_words(const int8_t* q, int u, int (&a)[8]) {
    const uint4 lo = lds128(q + 32 * u), hi = lds128(q + 32 * u + 16);
    a[0] = int(lo.x); a[1] = int(lo.y); a[2] = int(lo.z); a[3] = int(lo.w);
    a[4] = int(hi.x); a[5] = int(hi.y); a[6] = int(hi.z); a[7] = int(hi.w);
}
__device__ __forceinline__ int dot4(const uint32_t* w, const int* a) {
    int s = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) s = __dp4a(int(w[i]), a[i], s);
    return s;
}
// The 4 bits (bit j = element j) spread to one byte each (0 or 1).
__device__ __forceinline__ uint32_t spread4(uint32_t nib) { return (nib * 0x00204081u) & 0x01010101u; }
// get_scale_min_k4 (fast/lil_math.cpp:139-149): 6-bit scale and min of sub-block j of a K-quant.
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t* q, int& sc, int& m) {
    if (j < 4) {
        sc = q[j] & 63;
        m = q[j + 4] & 63;
    } else {
        sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}
// 6-bit scale of 16-element group g of a Q3_K block (the expansion at fast/lil_math.cpp:520-525),
// minus 32.
__device__ __forceinline__ int q3k_scale(const uint8_t* sb, int g) {
    const int i = g & 3;
    const int hi = (sb[8 + i] >> (2 * (g >> 2))) & 3;
    const int lo = (g & 4) ? sb[4 + i] : sb[i];
    return (((g & 8) ? (lo >> 4) : (lo & 0xF)) | (hi << 4)) - 32;
}

// A unit's weights, unpacked once (load) and dotted with any number of tokens' activations (dot).
template <int TY>
struct WUnit;

// F32 (dot_f32): 32 fp32 weights against the fp32 activation.
template <>
struct WUnit<QT_F32> {
    float w[32];
    __device__ __forceinline__ void load(const uint8_t* row, int u) {
        const float4* p = reinterpret_cast<const float4*>(row + 128 * u);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 v = p[i];
            w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
        }
    }
    __device__ __forceinline__ float dot(const QmvActView& A, int u) const {
        const float4* x = reinterpret_cast<const float4*>(A.xf + 32 * u);
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 b = x[i];
            s = fmaf(w[4 * i], b.x, s);
            s = fmaf(w[4 * i + 1], b.y, s);
            s = fmaf(w[4 * i + 2], b.z, s);
            s = fmaf(w[4 * i + 3], b.w, s);
        }
        return s;
    }
};
// F16 (dot_f16_f32).
template <>
struct WUnit<QT_F16> {
    float w[32];
    __device__ __forceinline__ void load(const uint8_t* row, int u) {
        const uint4* p = reinterpret_cast<const uint4*>(row + 64 * u);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint4 r = p[i];
            const uint32_t ww[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&ww[k]));
                w[8 * i + 2 * k] = f.x;
                w[8 * i + 2 * k + 1] = f.y;
            }
        }
    }
    __device__ __forceinline__ float dot(const QmvActView& A, int u) const {
        const float4* x = reinterpret_cast<const float4*>(A.xf + 32 * u);
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 b = x[i];
            s = fmaf(w[4 * i], b.x, s);
            s = fmaf(w[4 * i + 1], b.y, s);
            s = fmaf(w[4 * i + 2], b.z, s);
            s = fmaf(w[4 * i + 3], b.w, s);
        }
        return s;
    }
};
// Q8_0 (dot_q8_0_q8_0): block = unit, {fp16 d, int8 qs[32]}.
template <>
struct WUnit<QT_Q8_0> {
    uint32_t w[8];
    float d;
    __device__ __forceinline__ void load(const uint8_t* row, int u) {
        const uint8_t* blk = row + 34 * u;
        load8_a2(blk + 2, w);
        d = h2f(lds16(blk));
    }
    __device__ __forceinline__ float dot(const QmvActView& A, int u) const {
        int a[8];
        act_words(A.q0, u, a);
        return d * A.d0[u] * static_cast<float>(dot4(w, a) + dot4(w + 4, a + 4));
    }
};
// Q8_0 repacked at upload (rows of a multiple of 1024 elements): per group of 32 units (32
// blocks, 1088 bytes, as many as in the GGUF layout) the 32 x 32 int8 values first, then the 32
// fp16 scales, so a unit's values are two aligned 16-byte loads instead of nine 4-byte loads and
// eight funnel shifts of a 2-byte aligned block.  Same values, same dot.
template <>
struct WUnit<QT_Q8_0_G32> {
    uint32_t w[8];
    float d;
    __device__ __forceinline__ void load(const uint8_t* row, int u) {
        const uint8_t* grp = row + 1088 * (u >> 5);
        load8_a16(grp + 32 * (u & 31), w);
        d = h2f(lds16(grp + 1024 + 2 * (u & 31)));
    }
    __device__ __forceinline__ float dot(const QmvActView& A, int u) const {
        int a[8];
        act_words(A.q0, u, a);
        return d * A.d0[u] * static_cast<float>(dot4(w, a) + dot4(w + 4, a + 4));
    }
};
// The repack: GGUF Q8_0 rows (src) -> groups of 32 blocks as above (dst), one thread per block.
__global__ void __launch_bounds__(256) repack_q80_g32_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                                            size_t n_blocks) {
    const size_t b = blockIdx.x * size_t(256) + threadIdx.x;
    if (b >= n_blocks) return;
    const uint8_t* blk = src + 34 * b;
    uint8_t* grp = dst + 1088 * (b >> 5);
    const int j = int(b & 31);
    for (int i = 0; i < 32; ++i) grp[32 * j + i] = blk[2 + i];
    grp[1024 + 2 * j] = blk[0];
    grp[1024 + 2 * j + 1] = blk[1];
}
// Q1_0 (dot_q8_0_q1_0): block = unit, {fp16 d, 32 sign bits}; weight = bit ? +1 : -1, so the dot is
// 2 * (sum of x where the bit is set) - (sum of all x).
__device__ __forceinline__ int sign_dot(const uint32_t* w, const int* a) {
    int pos = 0, all = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        pos = __dp4a(int(w[i]), a[i], pos);
        all = __dp4a(0x01010101, a[i], all);
    }
    return 2 * pos - all;
}
template <>
struct WUnit<QT_Q1_0> {
    uint32_t w[8];
    float d;
    __device__ __forceinline__ void load(const uint8_t* row, int u) {
        const uint8_t* blk = row + 6 * u;
        const uint32_t bits = uint32_t(lds16(blk + 2)) | (uint32_t(lds16(blk + 4)) << 16);
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = spread4((bits >> (4 * i)) & 0xFu);
        d = h2f(lds16(blk));
    }
    __device__ __forceinline__ float dot(const QmvActView& A, int u) const {
        int a[8];
        act_words(A.q0, u, a);
        return d * A.d0[u] * static_cast<float>(sign_dot(w, a));
    }
};
// Q1_G (dot_q8_0_q1_G): block of 128 = 4 units, {fp16 d, 128 sign bits}.
template <>
struct WUnit<QT_Q1_G> {
    uint32_t w[8];
    float d;
    __device__ __forceinline__ void load(const uint8_t* row, int u) {
        const uint8_t* blk = row + 18 * (u >> 2);
        const uint8_t* qb = blk + 2 + 4 * (u & 3);
        const uint32_t bits = uint32_t(lds16(qb)) | (uint32_t(lds16(qb + 2)) << 16);
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = spread4((bits >> (4 * i)) & 0xFu);
        d = h2f(lds16(blk));
    }
    __device__ __forceinline__ float dot(const QmvActView& A, int u) const {
        int a[8];
        act_words(A.q0, u, a);
        return d * (A.d0[u] * static_cast<float>(sign_dot(w, a)));
    }
};
// Q2_K (dot_q8_K_q2_K): {scales[16] (4-bit scale | 4-bit min << 4), qs[64] 2-bit, fp16 d, dmin}.
template <>
struct WUnit<QT_Q2_K> {
    uint32_t w[8];
    int sc0, sc1, m0, m1;
    float d, dmin;
    __device__ __forceinline__ void load(const uint8_t* row, int u) {
        const int s = u & 7;
        const uint8_t* blk = row + 84 * (u >> 3);
        load8_a4(blk + 16 + 32 * (s >> 2), w);
        const int sh = 2 * (s & 3);
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = (w[i] >> sh) & 0x03030303u;
        const int b0 = blk[2 * s], b1 = blk[2 * s + 1];
        sc0 = b0 & 0xF; sc1 = b1 & 0xF; m0 = b0 >> 4; m1 = b1 >> 4;
        d = h2f(lds16(blk + 80));
        dmin = h2f(lds16(blk + 82));
    }
    __device__ __forceinline__ float dot(const QmvActView& A, int u) const {
        int a[8];
        act_words(A.qk, u, a);
        const int isum = sc0 * dot4(w, a) + sc1 * dot4(w + 4, a + 4);
        const int msum = m0 * A.bs[2 * u] + m1 * A.bs[2 * u + 1];
        const float dk = A.dk[u >> 3];
        return dk * d * static_cast<float>(isum) - dk * dmin * static_cast<float>(msum);
    }
};
// Q3_K (dot_q8_K_q3_K): {hmask[32], qs[64] 2-bit, scales[12], fp16 d}; value = q - 4 unless its
// hmask bit is set (held here as q | h << 2, minus 4 through the 16-element sums).
template <>
struct WUnit<QT_Q3_K> {
    uint32_t w[8];
    int s0, s1;
    float d;
    __device__ __forceinline__ void load(const uint8_t* row, int u) {
        const int s = u & 7, k = s >> 2, j = s & 3;
        const uint8_t* blk = row + 110 * (u >> 3);
        uint32_t h[8];
        load8_a2(blk + 32 + 32 * k, w);
        load8_a2(blk, h);
        const int hb = 4 * k + j;
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = ((w[i] >> (2 * j)) & 0x03030303u) | (((h[i] >> hb) & 0x01010101u) << 2);
        s0 = q3k_scale(blk + 96, 2 * s);
        s1 = q3k_scale(blk + 96, 2 * s + 1);
        d = h2f(lds16(blk + 108));
    }
    __device__ __forceinline__ float dot(const QmvActView& A, int u) const {
        int a[8];
        act_words(A.qk, u, a);
        const int i0 = dot4(w, a) - 4 * A.bs[2 * u];
        const int i1 = dot4(w + 4, a + 4) - 4 * A.bs[2 * u + 1];
        return d * A.dk[u >> 3] * static_cast<float>(s0 * i0 + s1 * i1);
    }
};
// Q4_K (dot_q8_K_q4_K): {fp16 d, dmin, scales[12], qs[128] nibbles}.
template <>
struct WUnit<QT_Q4_K> {
    uint32_t w[8];
    int sc, m;
    float d, dmin;
    __device__ __forceinline__ void load(const uint8_t* row, int u) {
        const int s = u & 7;
        const uint8_t* blk = row + 144 * (u >> 3);
        load8_a16(blk + 16 + 32 * (s >> 1), w);  // 144-byte blocks: 16-byte aligned
        const int sh = 4 * (s & 1);
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = (w[i] >> sh) & 0x0F0F0F0Fu;
        scale_min_k4(s, blk + 4, sc, m);
        d = h2f(lds16(blk));
        dmin = h2f(lds16(blk + 2));
    }
    __device__ __forceinline__ float dot(const QmvActView& A, int u) const {
        int a[8];
        act_words(A.qk, u, a);
        const int dt = dot4(w, a) + dot4(w + 4, a + 4);
        const float dk = A.dk[u >> 3];
        return d * dk * static_cast<float>(sc) * static_cast<float>(dt) -
               dmin * dk * static_cast<float>(m) * static_cast<float>(A.bs[2 * u] + A.bs[2 * u + 1]);
    }
};
// Q5_K (dot_q8_K_q5_K): {fp16 d, dmin, scales[12], qh[32] fifth bits, qs[128] nibbles}.
template <>
struct WUnit<QT_Q5_K> {
    uint32_t w[8];
    int sc, m;
    float d, dmin;
    __device__ __forceinline__ void load(const uint8_t* row, int u) {
        const int s = u & 7;
        const uint8_t* blk = row + 176 * (u >> 3);
        uint32_t h[8];
        load8_a16(blk + 48 + 32 * (s >> 1), w);  // 176-byte blocks: 16-byte aligned
        load8_a16(blk + 16, h);
        const int sh = 4 * (s & 1);
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = ((w[i] >> sh) & 0x0F0F0F0Fu) | (((h[i] >> s) & 0x01010101u) << 4);
        scale_min_k4(s, blk + 4, sc, m);
        d = h2f(lds16(blk));
        dmin = h2f(lds16(blk + 2));
    }
    __device__ __forceinline__ float dot(const QmvActView& A, int u) const {
        int a[8];
        act_words(A.qk, u, a);
        const int dt = dot4(w, a) + dot4(w + 4, a + 4);
        const float dk = A.dk[u >> 3];
        return d * dk * static_cast<float>(sc * dt) - dmin * dk * static_cast<float>(m * (A.bs[2 * u] + A.bs[2 * u + 1]));
    }
};
// Q6_K (dot_q8_K_q6_K): {ql[128] low nibbles, qh[64] 2-bit highs, int8 scales[16], fp16 d};
// value = 6-bit q - 32 (held as q; the 32 comes off through the 16-element sums).
template <>
struct WUnit<QT_Q6_K> {
    uint32_t w[8];
    int s0, s1;
    float d;
    __device__ __forceinline__ void load(const uint8_t* row, int u) {
        const int s = u & 7, c = s >> 2, qq = s & 3;
        const uint8_t* blk = row + 210 * (u >> 3);
        uint32_t hi[8];
        load8_a2(blk + 64 * c + 32 * (qq & 1), w);
        load8_a2(blk + 128 + 32 * c, hi);
        const int lsh = 4 * (qq >> 1), hsh = 2 * qq;
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = ((w[i] >> lsh) & 0x0F0F0F0Fu) | (((hi[i] >> hsh) & 0x03030303u) << 4);
        const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192);
        s0 = sc[2 * s];
        s1 = sc[2 * s + 1];
        d = h2f(lds16(blk + 208));
    }
    __device__ __forceinline__ float dot(const QmvActView& A, int u) const {
        int a[8];
        act_words(A.qk, u, a);
        const int i0 = dot4(w, a) - 32 * A.bs[2 * u];
        const int i1 = dot4(w + 4, a + 4) - 32 * A.bs[2 * u + 1];
        return d * A.dk[u >> 3] * static_cast<float>(s0 * i0 + s1 * i1);
    }
};

// One tile of `nrows` rows (row stride rb) staged at `tile`: warp w takes rows w, w+kQmvWarps, ...;
// each lane a unit at a time, its weights unpacked once for the T tokens.
template <int TY, int T>
__device__ __forceinline__ void qmv_tile(const uint8_t* tile, int nrows, int rb, int units, const uint8_t* act,
                                         const QmvAct& L, int n_tok, float* out, long long out_stride, int warp,
                                         int lane, const QmvRed& red, int epoch, int r0, int rows) {
    for (int r = warp; r < nrows; r += kQmvWarps) {
        const uint8_t* row = tile + size_t(r) * rb;
        float acc[T];
#pragma unroll
        for (int t = 0; t < T; ++t) acc[t] = 0.f;
        for (int u = lane; u < units; u += 32) {
            WUnit<TY> wu;
            wu.load(row, u);
#pragma unroll
            for (int t = 0; t < T; ++t)
                if (t < n_tok) acc[t] += wu.dot(act_view(act, L, t), u);
        }
#pragma unroll
        for (int t = 0; t < T; ++t) {
            if (t < n_tok) {
                const float v = warp_sum(acc[t]);
                if (red.peers) {  // lane p stores to rank p's buffer
                    const unsigned long long w =
                        (static_cast<unsigned long long>(static_cast<uint32_t>(epoch)) << 32) | __float_as_uint(v);
                    const size_t e = (size_t(epoch & 1) * red.nranks + red.rank) * size_t(rows) + r0 + r;
                    for (int p = lane; p < red.nranks; p += 32)
                        asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(red.peers[p] + e), "l"(w) : "memory");
                } else if (lane == 0) {
                    out[t * out_stride + r] = v;
                }
            }
        }
    }
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ int qmv_find_mat(const QmvArgs& a, int t) {
    int m = 0;
    while (m + 1 < a.nmat && t >= a.m[m + 1].tile0) ++m;
    return m;
}

template <int T>
__global__ void __launch_bounds__(kQmvThreads, 2) qmv_kernel(const __grid_constant__ QmvArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* ring = smem + a.act.bytes;
    __shared__ uint64_t full[kQmvMaxStages], empty[kQmvMaxStages];
    const int S = a.stages;
    __shared__ int abort_s;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t_begin = int((long long)blockIdx.x * a.ntiles / gridDim.x);
    const int t_end = int((long long)(blockIdx.x + 1) * a.ntiles / gridDim.x);
    const uint64_t deadline = globaltimer_ns() + kWaitLimitNs;
    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kQmvWarps);
        }
        abort_s = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kQmvWarps) {  // ------------------------------------------------ producer
        if (lane == 0) {
            int issued = 0;
            for (int t = t_begin, it = 0; t < t_end; ++t, ++it) {
                const int s = it % S;
                if (it >= S &&
                    !mbar_wait_bounded(&empty[s], ((it / S) - 1) & 1, deadline, &abort_s)) {
                    abort_s = 1;
                    *reinterpret_cast<volatile int*>(a.err) = KERR_TIMEOUT_EMPTY;
                    break;
                }
                const QmvMat& m = a.m[qmv_find_mat(a, t)];
                const int r0 = (t - m.tile0) * m.tile_rows;
                const int nrows = min(m.tile_rows, m.rows - r0);
                const uint32_t bytes = (uint32_t(nrows) * m.rb + 15u) & ~15u;
                mbar_arrive_expect_tx(&full[s], bytes);
                bulk_load(ring + s * kQmvStageMax, m.w + size_t(r0) * m.rb, bytes, &full[s]);
                ++issued;
            }
            // the copies must land before the CTA exits (bounded, past the consumers' deadline)
            const uint64_t dd = deadline + kWaitLimitNs / 2;
            for (int u = max(0, issued - S); u < issued; ++u)
                while (!mbar_try_wait(&full[u % S], (u / S) & 1) && globaltimer_ns() < dd) {
                }
        }
        return;
    }

    // ------------------------------------------------------------------------- consumers
    asm volatile("griddepcontrol.wait;" ::: "memory");  // x comes from the previous kernel
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (a.act_g) {
        // The tokens' activation forms, quantized once for the call by qmv_act_kernel (from L2).
        const uint4* src = reinterpret_cast<const uint4*>(a.act_g);
        uint4* dst = reinterpret_cast<uint4*>(smem);
        const int n16 = a.n_tok * a.act.tok_bytes / 16;
        for (int i = tid; i < n16; i += kQmvWarps * 32) dst[i] = __ldcg(src + i);
    } else {
        // One token: its forms here, in each CTA, which costs less than another launch.  Q8_K: a
        // warp per 256-element block; Q8_0: a lane per 32-element block (no shuffles: 128 blocks of a
        // 4096-wide x are one pass of 4 warps); the fp32 copy for F32/F16 weights.
        if (a.need_k)
            for (int b = warp; b < a.n / 256; b += kQmvWarps)
                q8k_block_warp(a.x + 256 * b, reinterpret_cast<int8_t*>(smem + a.act.off_qk) + 256 * b,
                               reinterpret_cast<float*>(smem + a.act.off_dk) + b,
                               reinterpret_cast<int*>(smem + a.act.off_bs) + 16 * b, nullptr, lane);
        if (a.need_0)
            for (int b = tid; b < a.n / 32; b += kQmvWarps * 32)
                q80_block_lane(a.x + 32 * b, reinterpret_cast<int8_t*>(smem + a.act.off_q0) + 32 * b,
                               reinterpret_cast<float*>(smem + a.act.off_d0) + b);
        if (a.need_f) {
            const float4* x4 = reinterpret_cast<const float4*>(a.x);
            float4* dst = reinterpret_cast<float4*>(smem + a.act.off_xf);
            for (int i = tid; i < a.n / 4; i += kQmvWarps * 32) dst[i] = x4[i];
        }
    }
    named_bar_sync(1, kQmvWarps * 32);
    const int epoch = a.red.peers ? __ldcg(a.red.state) + 1 : 0;

    const int units = a.n / 32;
    for (int t = t_begin, it = 0; t < t_end; ++t, ++it) {
        const int s = it % S;
        const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(&full[s], (it / S) & 1, deadline, &abort_s));
        if (!ok) {
            if (lane == 0) {
                abort_s = 1;
                *reinterpret_cast<volatile int*>(a.err) = KERR_TIMEOUT_FULL;
            }
            break;
        }
        const QmvMat& m = a.m[qmv_find_mat(a, t)];
        const int r0 = (t - m.tile0) * m.tile_rows;
        const int nrows = min(m.tile_rows, m.rows - r0);
        const uint8_t* tile = ring + s * kQmvStageMax;
        float* out = m.out + r0;
#define LG_QMV_CASE(TY)                                                                                    \
    case TY:                                                                                               \
        qmv_tile<TY, T>(tile, nrows, m.rb, units, smem, a.act, a.n_tok, out, m.out_stride, warp, lane, a.red, \
                        epoch, r0, m.rows);                                                                \
        break;
        switch (m.type) {
            LG_QMV_CASE(QT_F32)
            LG_QMV_CASE(QT_F16)
            LG_QMV_CASE(QT_Q8_0)
            LG_QMV_CASE(QT_Q8_0_G32)
            LG_QMV_CASE(QT_Q1_0)
            LG_QMV_CASE(QT_Q1_G)
            LG_QMV_CASE(QT_Q2_K)
            LG_QMV_CASE(QT_Q3_K)
            LG_QMV_CASE(QT_Q4_K)
            LG_QMV_CASE(QT_Q5_K)
            default:
                qmv_tile<QT_Q6_K, T>(tile, nrows, m.rb, units, smem, a.act, a.n_tok, out, m.out_stride, warp, lane,
                                     a.red, epoch, r0, m.rows);
        }
#undef LG_QMV_CASE
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
}

// Reduce wait (the SARA master's sum, cpp/ligguf_distrib.cpp:1040-1045, for every rank at once): one
// thread per row polls the row's word of every rank in this rank's buffer until each carries the
// call's epoch (bounded), sums them in rank order (rank 0's partial, then += rank 1's, ...), and adds
// the sum to the residual x (fast/ligguf_fast_qk.cpp:111: x += attention output) and/or writes it to
// `out`.  Epoch = state[0] + 1; the last block to finish advances state[0] (state[1] counts blocks).
// Launched after the projection; it starts while the projection runs (its only inputs from it are
// the self-validating words).
__global__ void __launch_bounds__(256) reduce_wait_kernel(const unsigned long long* buf, int* state, int nranks,
                                                          int rows, float* x_inout, float* out, int* err) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int epoch = __ldcg(state) + 1;
    const unsigned long long* slot = buf + size_t(epoch & 1) * nranks * rows;
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r < rows) {
        const uint64_t deadline = globaltimer_ns() + kWaitLimitNs;
        const uint32_t want = static_cast<uint32_t>(epoch);
        float sum = 0.f;
        bool ok = true;
        for (int p = 0; p < nranks && ok; ++p) {
            unsigned long long w;
            uint32_t spins = 0;
            while (true) {
                asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(slot + size_t(p) * rows + r) : "memory");
                if (static_cast<uint32_t>(w >> 32) == want) break;
                if ((++spins & 63u) == 0u && globaltimer_ns() > deadline) {
                    *reinterpret_cast<volatile int*>(err) = KERR_TIMEOUT_PEER;
                    ok = false;
                    break;
                }
            }
            const float v = __uint_as_float(static_cast<uint32_t>(w));
            sum = p == 0 ? v : __fadd_rn(sum, v);
        }
        if (ok) {
            if (out) out[r] = sum;
            if (x_inout) x_inout[r] = __fadd_rn(x_inout[r], sum);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(&state[1], 1) == static_cast<int>(gridDim.x) - 1) {
        state[1] = 0;
        state[0] = epoch;
    }
}

// Activation quantizers on their own, writing the reference's block layouts: block_q8_K
// {float d; int8 qs[256]; int16 bsums[16]} (292 bytes) and block_q8_0 {fp16 d; int8 qs[32]}
// (34 bytes).  One warp per block.
// The activation forms of n_tok tokens, once per call (the reference quantizes x once and then
// runs the matmuls, fast/lil_math.cpp:827-899): Q8_K blocks, Q8_0 blocks and/or the fp32 copy,
// in the QmvAct layout of the projection kernel's shared memory, into `out` (tok_bytes per token).
// One warp per work item: a Q8_K block, a Q8_0 block or 256 floats of the copy.  A programmatic
// dependent of the kernel that wrote x; the projection kernel that follows is one of this kernel
// and starts streaming its weights while this one runs.
struct QmvActArgs {
    const float* x;  // x[t * x_stride + i], t < n_tok
    long long x_stride;
    int n_tok, n;
    int need_k, need_0, need_f;
    QmvAct act;
    uint8_t* out;
};
__host__ __device__ inline int qmv_act_items(const QmvActArgs& a) {
    return a.n_tok * ((a.need_k ? a.n / 256 : 0) + (a.need_0 ? a.n / 32 : 0) + (a.need_f ? (a.n + 255) / 256 : 0));
}
__global__ void __launch_bounds__(256) qmv_act_kernel(const __grid_constant__ QmvActArgs a) {
    asm volatile("griddepcontrol.wait;" ::: "memory");  // x comes from the previous kernel
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int item = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    const int nk = a.need_k ? a.n / 256 : 0, n0 = a.need_0 ? a.n / 32 : 0, nf = a.need_f ? (a.n + 255) / 256 : 0;
    const int per_tok = nk + n0 + nf;
    if (item >= a.n_tok * per_tok) return;
    const int t = item / per_tok;
    int r = item - t * per_tok;
    const float* x = a.x + t * a.x_stride;
    uint8_t* tb = a.out + size_t(t) * a.act.tok_bytes;
    if (r < nk) {
        q8k_block_warp(x + 256 * r, reinterpret_cast<int8_t*>(tb + a.act.off_qk) + 256 * r,
                       reinterpret_cast<float*>(tb + a.act.off_dk) + r, reinterpret_cast<int*>(tb + a.act.off_bs) + 16 * r,
                       nullptr, lane);
        return;
    }
    r -= nk;
    if (r < n0) {
        uint16_t dh;
        const int q = q80_block_warp(x[32 * r + lane], &dh, lane);
        reinterpret_cast<int8_t*>(tb + a.act.off_q0)[32 * r + lane] = static_cast<int8_t>(q);
        if (lane == 0) reinterpret_cast<float*>(tb + a.act.off_d0)[r] = h2f(dh);
        return;
    }
    r -= n0;  // floats [256 r, 256 r + 256) of the copy (n is a multiple of 4)
    const float4* src = reinterpret_cast<const float4*>(x);
    float4* dst = reinterpret_cast<float4*>(tb + a.act.off_xf);
    for (int i = 64 * r + lane; i < min(64 * r + 64, a.n / 4); i += 32) dst[i] = src[i];
}

__global__ void __launch_bounds__(256) quantize_q8k_kernel(const float* __restrict__ x, int nblocks, uint8_t* out) {
    const int b = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (b >= nblocks) return;
    __shared__ __align__(16) int8_t q[8][256];
    __shared__ int16_t bs[8][16];
    __shared__ float d[8];
    const int w = threadIdx.x >> 5;
    q8k_block_warp(x + 256 * size_t(b), q[w], &d[w], nullptr, bs[w], lane);
    __syncwarp();
    uint8_t* o = out + size_t(b) * 292;
    if (lane == 0) *reinterpret_cast<float*>(o) = d[w];
    for (int i = lane; i < 256; i += 32) o[4 + i] = static_cast<uint8_t>(q[w][i]);
    if (lane < 16) *reinterpret_cast<int16_t*>(o + 260 + 2 * lane) = bs[w][lane];
}
__global__ void __launch_bounds__(256) quantize_q80_kernel(const float* __restrict__ x, int nblocks, uint8_t* out) {
    const int b = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (b >= nblocks) return;
    uint16_t dh;
    const int q = q80_block_warp(x[32 * size_t(b) + lane], &dh, lane);
    uint8_t* o = out + size_t(b) * 34;
    o[2 + lane] = static_cast<uint8_t>(static_cast<int8_t>(q));
    if (lane == 0) {
        o[0] = static_cast<uint8_t>(dh & 0xFF);
        o[1] = static_cast<uint8_t>(dh >> 8);
    }
}

}  // namespace lg
