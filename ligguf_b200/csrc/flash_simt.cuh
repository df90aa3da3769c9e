// flash_simt.cuh - fp32 tiled attention on CUDA cores for many query rows at once: causal prefill
// over the KV cache and the BERT embedding attention.  This is the tight-tolerance path (every
// product and sum in fp32, expf for the exponentials); the tensor-core path is flash_tc.cuh.
//
// Semantics:
//   prefill: fast/ligguf_fast_qk.cpp:340-356 runs inference() once per prompt token, so query
//            row r (absolute position q_pos0 + r) attends keys t <= q_pos0 + r of the cache,
//            scores scaled like fast/ligguf_fast_qk.cpp:85, softmax fast/lil_math.cpp:964-976.
//   BERT:    fast/vdb.cpp:189-212: every token of a sequence attends every token of the same
//            sequence (no causal mask); sequences are batched here with per-sequence lengths.
//
// CTA = (64 query rows, one q head, one batch entry), 256 threads.  Keys/values stream through
// shared memory 32 rows at a time (converted to fp32 from the cache type on load), scores and
// P.V use 4x2 / 4x8 register tiles per thread, softmax is online (running max and sum per row).
#pragma once

#include "common.cuh"
#include "decode.cuh"  // norm_rope_head

namespace lg {

struct FlashArgs {
    const float* q;        // query rows, fp32; element (b, r, h, d) at q[b*q_batch + r*q_row + h*D + d]
    long long q_row, q_batch;
    const void* k;         // keys (KV type); element (b, t, g, d) at k[b*kv_batch + t*kv_row + g*D + d]
    const void* v;
    long long kv_row, kv_batch;
    float* out;            // element (b, r, h, d) at out[b*o_batch + r*o_row + h*D + d]
    long long o_row, o_batch;
    const int* lens;       // per-batch valid rows (query and key) or null
    int n_q;               // query rows per batch entry
    int kv_len;            // keys per batch entry when lens == null
    int causal;
    int q_pos0;            // absolute position of query row 0 (causal mask: t <= q_pos0 + r)
    int nrep;              // q heads per kv head
    int scale_div;
    float scale;
};

constexpr int kFlashBQ = 64;
constexpr int kFlashBK = 32;
constexpr int kFlashThreads = 256;

template <int D>
struct FlashSimtSmem {
    static constexpr int kQP = D + 4;  // padded row pitch (floats): conflict-free float4 reads
    static constexpr int kKP = D + 4;
    static constexpr int kVP = D;
    static constexpr int kPP = kFlashBK + 1;
    static constexpr size_t kFloats =
        size_t(kFlashBQ) * kQP + size_t(kFlashBK) * kKP + size_t(kFlashBK) * kVP + size_t(kFlashBQ) * kPP;
    static constexpr size_t kBytes = kFloats * 4;
};

template <typename KV, int D>
__global__ void __launch_bounds__(kFlashThreads) flash_simt_kernel(const FlashArgs a) {
    using Sm = FlashSimtSmem<D>;
    constexpr int BQ = kFlashBQ, BK = kFlashBK;
    constexpr int QP = Sm::kQP, KP = Sm::kKP, VP = Sm::kVP, PP = Sm::kPP;
    constexpr int OC = D / 16;  // output columns per thread: 4*tx + 64*c + e
    constexpr int EPV = KvTraits<KV>::kElemsPer16B;
    extern __shared__ __align__(16) float fsm[];
    float* Qs = fsm;
    float* Ks = Qs + BQ * QP;
    float* Vs = Ks + BK * KP;
    float* Ps = Vs + BK * VP;

    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int g = h / a.nrep;
    const int nq_valid = a.lens ? min(a.lens[b], a.n_q) : a.n_q;
    const int kv_end = a.lens ? a.lens[b] : a.kv_len;
    const int r0 = qt * BQ;
    const float* qb = a.q + b * a.q_batch + static_cast<long long>(h) * D;
    float* ob = a.out + b * a.o_batch + static_cast<long long>(h) * D;
    const KV* kb = reinterpret_cast<const KV*>(a.k) + b * a.kv_batch + static_cast<long long>(g) * D;
    const KV* vb = reinterpret_cast<const KV*>(a.v) + b * a.kv_batch + static_cast<long long>(g) * D;

    if (r0 >= nq_valid) {  // padded query rows: zeros
        for (int idx = tid; idx < BQ * D; idx += kFlashThreads) {
            const int r = r0 + idx / D;
            if (r < a.n_q) ob[r * a.o_row + idx % D] = 0.f;
        }
        return;
    }

    for (int idx = tid; idx < BQ * (D / 4); idx += kFlashThreads) {
        const int r = idx / (D / 4), c4 = idx % (D / 4);
        float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r0 + r < nq_valid) val = *reinterpret_cast<const float4*>(qb + (r0 + r) * a.q_row + 4 * c4);
        *reinterpret_cast<float4*>(Qs + r * QP + 4 * c4) = val;
    }

    int kv_stop = kv_end;
    if (a.causal) kv_stop = min(kv_stop, a.q_pos0 + min(r0 + BQ, nq_valid));

    float m[4], l[4], o[4][OC];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.f;
#pragma unroll
        for (int c = 0; c < OC; ++c) o[i][c] = 0.f;
    }
    const bool div = a.scale_div != 0;

    for (int k0 = 0; k0 < kv_stop; k0 += BK) {
        __syncthreads();  // previous tile fully consumed
        for (int idx = tid; idx < BK * (D / EPV); idx += kFlashThreads) {
            const int t = idx / (D / EPV), cv = idx % (D / EPV);
            float kx[EPV], vx[EPV];
            if (k0 + t < kv_stop) {
                const uint4 kr = *reinterpret_cast<const uint4*>(kb + (k0 + t) * a.kv_row + cv * EPV);
                const uint4 vr = *reinterpret_cast<const uint4*>(vb + (k0 + t) * a.kv_row + cv * EPV);
                KvTraits<KV>::unpack(kr, kx);
                KvTraits<KV>::unpack(vr, vx);
            } else {
#pragma unroll
                for (int e = 0; e < EPV; ++e) kx[e] = vx[e] = 0.f;
            }
#pragma unroll
            for (int e = 0; e < EPV; ++e) {
                Ks[t * KP + cv * EPV + e] = kx[e];
                Vs[t * VP + cv * EPV + e] = vx[e];
            }
        }
        __syncthreads();

        float s[4][2];
#pragma unroll
        for (int i = 0; i < 4; ++i) s[i][0] = s[i][1] = 0.f;
#pragma unroll 4
        for (int d = 0; d < D; d += 4) {
            float4 qv[4], kv[2];
#pragma unroll
            for (int i = 0; i < 4; ++i) qv[i] = *reinterpret_cast<const float4*>(Qs + (ty + 16 * i) * QP + d);
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) kv[jj] = *reinterpret_cast<const float4*>(Ks + (tx + 16 * jj) * KP + d);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int jj = 0; jj < 2; ++jj) {
                    float acc = s[i][jj];
                    acc = fmaf(qv[i].x, kv[jj].x, acc);
                    acc = fmaf(qv[i].y, kv[jj].y, acc);
                    acc = fmaf(qv[i].z, kv[jj].z, acc);
                    acc = fmaf(qv[i].w, kv[jj].w, acc);
                    s[i][jj] = acc;
                }
        }

#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = r0 + ty + 16 * i;
            float mx = -INFINITY;
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
                const int t = k0 + tx + 16 * jj;
                const bool valid = t < kv_stop && r < nq_valid && (!a.causal || t <= a.q_pos0 + r);
                s[i][jj] = valid ? (div ? s[i][jj] / a.scale : s[i][jj] * a.scale) : -INFINITY;
                mx = fmaxf(mx, s[i][jj]);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float m_new = fmaxf(m[i], mx);
            float corr = 1.f, rs = 0.f;
            float p[2] = {0.f, 0.f};
            if (m_new != -INFINITY) {
                corr = expf(m[i] - m_new);
#pragma unroll
                for (int jj = 0; jj < 2; ++jj) {
                    p[jj] = expf(s[i][jj] - m_new);
                    rs += p[jj];
                }
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
            l[i] = l[i] * corr + rs;
            m[i] = m_new;
#pragma unroll
            for (int c = 0; c < OC; ++c) o[i][c] *= corr;
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) Ps[(ty + 16 * i) * PP + tx + 16 * jj] = p[jj];
        }
        __syncthreads();

#pragma unroll 4
        for (int kk = 0; kk < BK; ++kk) {
            float p[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) p[i] = Ps[(ty + 16 * i) * PP + kk];
#pragma unroll
            for (int c = 0; c < OC / 4; ++c) {
                const float4 vv = *reinterpret_cast<const float4*>(Vs + kk * VP + 4 * tx + 64 * c);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    o[i][4 * c + 0] = fmaf(p[i], vv.x, o[i][4 * c + 0]);
                    o[i][4 * c + 1] = fmaf(p[i], vv.y, o[i][4 * c + 1]);
                    o[i][4 * c + 2] = fmaf(p[i], vv.z, o[i][4 * c + 2]);
                    o[i][4 * c + 3] = fmaf(p[i], vv.w, o[i][4 * c + 3]);
                }
            }
        }
    }

#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = r0 + ty + 16 * i;
        if (r >= a.n_q) continue;
        float* orow = ob + r * a.o_row;
        if (r < nq_valid) {
            const float inv = 1.0f / l[i];
#pragma unroll
            for (int c = 0; c < OC / 4; ++c)
                *reinterpret_cast<float4*>(orow + 4 * tx + 64 * c) =
                    make_float4(o[i][4 * c] * inv, o[i][4 * c + 1] * inv, o[i][4 * c + 2] * inv,
                                o[i][4 * c + 3] * inv);
        } else {
#pragma unroll
            for (int c = 0; c < OC / 4; ++c)
                *reinterpret_cast<float4*>(orow + 4 * tx + 64 * c) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
}

// ------------------------------------------------------------------------------------- prep
// Prefill prologue: QK norm + RoPE for n tokens, append k, v to cache rows [pos0, pos0+n), and
// write the attention operands: fp32 q rows (SIMT path) or bf16 q/k/v (tensor-core path).
struct PrepArgs {
    const float* q;   // [n][q_headn*D] raw
    const float* k;   // [n][kv_headn*D]
    const float* v;
    const float* qg;
    const float* kg;
    const float* freq;
    void* kc;         // this layer's cache block
    void* vc;
    float* qf;        // [n][q_headn*D] fp32 out (or null)
    __nv_bfloat16* qb;  // [n][q_headn*D] bf16 out (or null)
    __nv_bfloat16* kb;  // [n_context][kv_dim] bf16 key shadow, rows by absolute position (or null)
    __nv_bfloat16* vb;
    int* wm;            // the layer's shadow watermark: shadow rows [0, *wm) equal the cache rows
    int* err;           // error word (mapped host memory): set when the row copies did not land
    int n, pos0, q_headn, kv_headn, kv_dim, rope_pairs, qk_norm;
    float eps;
};

// E = 2 or 4 consecutive floats of one lane: loads and stores of one row segment.
template <int E>
__device__ __forceinline__ void load_vec(const float* p, float (&x)[E]) {
    if constexpr (E == 4) {
        const float4 v = *reinterpret_cast<const float4*>(p);
        x[0] = v.x, x[1] = v.y, x[2] = v.z, x[3] = v.w;
    } else {
        const float2 v = *reinterpret_cast<const float2*>(p);
        x[0] = v.x, x[1] = v.y;
    }
}
template <int E>
__device__ __forceinline__ void store_vec_f32(float* p, const float (&x)[E]) {
    if constexpr (E == 4)
        *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
    else
        *reinterpret_cast<float2*>(p) = make_float2(x[0], x[1]);
}
// Two floats as one 32-bit word of 16-bit values of type T (lower element in the low half).
template <typename T>
__device__ __forceinline__ uint32_t pack16(float x, float y) {
    const T lo = KvTraits<T>::from_float(x), hi = KvTraits<T>::from_float(y);
    return uint32_t(*reinterpret_cast<const uint16_t*>(&lo)) | (uint32_t(*reinterpret_cast<const uint16_t*>(&hi)) << 16);
}
template <typename T, int E>
__device__ __forceinline__ void store_vec16(T* p, const float (&x)[E]) {
    if constexpr (E == 4)
        *reinterpret_cast<uint2*>(p) = make_uint2(pack16<T>(x[0], x[1]), pack16<T>(x[2], x[3]));
    else
        *reinterpret_cast<uint32_t*>(p) = pack16<T>(x[0], x[1]);
}
template <typename KV, int E>
__device__ __forceinline__ void store_vec_kv(KV* p, const float (&x)[E]) {
    if constexpr (sizeof(KV) == 4)
        store_vec_f32<E>(reinterpret_cast<float*>(p), x);
    else
        store_vec16<KV, E>(p, x);
}

// Qwen3 per-head RMS norm (with gamma) and RoPE of one head row held as E = D/32 consecutive
// elements per lane: elements [E*lane, E*lane + E), pairs m = lane*E/2 + i rotated by (cs[m], sn[m]).
// Same arithmetic as norm_rope_regs (sum of squares, 1/sqrt, gamma, rotation); only the partial
// sums of squares are formed in another order.
template <int D>
__device__ __forceinline__ void norm_rope_vec(float (&x)[D / 32], const float* __restrict__ gamma, int norm,
                                              float eps, const float* cs, const float* sn, int rope_pairs,
                                              int lane) {
    constexpr int E = D / 32;
    if (norm) {
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) ss = fmaf(x[e], x[e], ss);
        ss = warp_sum(ss);
        const float rs = 1.0f / sqrtf(ss / static_cast<float>(D) + eps);
        float g[E];
        load_vec<E>(gamma + lane * E, g);
#pragma unroll
        for (int e = 0; e < E; ++e) x[e] = (x[e] * rs) * g[e];
    }
#pragma unroll
    for (int i = 0; i < E / 2; ++i) {
        const int m = lane * (E / 2) + i;
        if (m < rope_pairs) {
            const float c = cs[m], sn_ = sn[m];
            const float x0 = x[2 * i], x1 = x[2 * i + 1];
            x[2 * i] = x0 * c - x1 * sn_;
            x[2 * i + 1] = x0 * sn_ + x1 * c;
        }
    }
}

// Prompt rows before attention: per token, the q heads (norm + RoPE; fp32 and/or bf16 out), the k
// heads (norm + RoPE) and the v heads into this layer's cache rows (and their bf16 shadow).  One
// block per token: thread 0 brings the token's q, k and v rows (24 KB for Qwen3-8B) into shared
// memory with three bulk copies, which need no registers, so 8 blocks of an SM keep twice the bytes
// in flight that register loads did (the kernel is bound by the bytes each SM keeps in flight);
// the RoPE rotation is computed while they land, then the heads are dealt to the warps (one warp
// per head, each lane E = D/32 consecutive elements).  q, k, v must be 16-byte aligned.
constexpr int kPrepWarps = 8;
template <typename KV, int D>
__global__ void __launch_bounds__(kPrepWarps * 32) prefill_prep_kernel(const PrepArgs a) {
    // Launched in stream order (its predecessor has completed); the tensor-core kernel that follows
    // is a programmatic dependent and may start its set-up once every block of this grid has begun.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    constexpr int E = D / 32;
    extern __shared__ __align__(16) float rows[];  // [q_headn + 2 * kv_headn][D] of this token
    __shared__ float cs[D / 2], sn[D / 2];          // RoPE rotation of this token, shared by all heads
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_s;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int i = blockIdx.x;
    const int pos = a.pos0 + i;
    const int n_jobs = a.q_headn + 2 * a.kv_headn;
    const uint32_t qbytes = uint32_t(a.q_headn) * D * 4, kbytes = uint32_t(a.kv_headn) * D * 4;
    if (threadIdx.x == 0) {
        abort_s = 0;
        mbar_init(&bar, 1);
        fence_mbar_init();
        mbar_arrive_expect_tx(&bar, qbytes + 2 * kbytes);
        bulk_copy_g2s(rows, a.q + static_cast<size_t>(i) * a.q_headn * D, qbytes, &bar);
        bulk_copy_g2s(rows + a.q_headn * D, a.k + static_cast<size_t>(i) * a.kv_headn * D, kbytes, &bar);
        bulk_copy_g2s(rows + (a.q_headn + a.kv_headn) * D, a.v + static_cast<size_t>(i) * a.kv_headn * D, kbytes,
                      &bar);
    }
    for (int m = threadIdx.x; m < a.rope_pairs; m += blockDim.x)
        sincosf(static_cast<float>(pos) * a.freq[m], &sn[m], &cs[m]);
    // Watermark: with shadows, rows [0, pos0) were brought up to date by shadow_sync_kernel and this
    // grid writes [pos0, pos0 + n) to both; without, the cache rows from pos0 up change under them.
    if (a.wm && i == 0 && threadIdx.x == 0)
        *a.wm = a.kb ? max(*a.wm, a.pos0 + a.n) : min(*a.wm, a.pos0);
    __syncthreads();  // the barrier's initialisation and the rotation are visible to every thread
    const uint64_t deadline = globaltimer_ns() + kWaitLimitNs;
    if (!mbar_wait_bounded(&bar, 0, deadline, &abort_s)) {
        abort_s = 1;
        if (a.err) *reinterpret_cast<volatile int*>(a.err) = KERR_TIMEOUT_FULL;
        // the copies write this block's shared memory: let them land (bounded) before exiting
        const uint64_t dd = deadline + kWaitLimitNs / 2;
        while (!mbar_try_wait(&bar, 0) && globaltimer_ns() < dd) {
        }
        return;
    }
    for (int job = warp; job < n_jobs; job += kPrepWarps) {
        const bool is_q = job < a.q_headn, is_k = !is_q && job < a.q_headn + a.kv_headn;
        const int gi = is_q ? job : (is_k ? job - a.q_headn : job - a.q_headn - a.kv_headn);
        float x[E];
        load_vec<E>(rows + job * D + lane * E, x);
        if (is_q) {
            norm_rope_vec<D>(x, a.qg, a.qk_norm, a.eps, cs, sn, a.rope_pairs, lane);
            const size_t o = (static_cast<size_t>(i) * a.q_headn + gi) * D + lane * E;
            if (a.qf) store_vec_f32<E>(a.qf + o, x);
            if (a.qb) store_vec16<__nv_bfloat16, E>(a.qb + o, x);
            continue;
        }
        if (is_k) norm_rope_vec<D>(x, a.kg, a.qk_norm, a.eps, cs, sn, a.rope_pairs, lane);
        const size_t o = static_cast<size_t>(pos) * a.kv_dim + static_cast<size_t>(gi) * D + lane * E;
        store_vec_kv<KV, E>(reinterpret_cast<KV*>(is_k ? a.kc : a.vc) + o, x);
        __nv_bfloat16* shadow = is_k ? a.kb : a.vb;
        if (shadow) store_vec16<__nv_bfloat16, E>(shadow + o, x);
    }
}

// Before a tensor-core prefill at pos0: the layer's cache rows [min(*wm, pos0), pos0) -> its bf16
// shadows, i.e. only the rows written since the shadows last matched the cache (none when a prompt
// is prefilled chunk after chunk with nothing else writing the cache in between).
template <typename KV>
__global__ void shadow_sync_kernel(const KV* __restrict__ kc, const KV* __restrict__ vc, __nv_bfloat16* __restrict__ kb,
                                   __nv_bfloat16* __restrict__ vb, int kv_dim, const int* __restrict__ wm, int pos0) {
    const size_t end = size_t(pos0) * kv_dim;
    for (size_t i = size_t(min(*wm, pos0)) * kv_dim + blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < end;
         i += size_t(gridDim.x) * blockDim.x) {
        kb[i] = __float2bfloat16_rn(KvTraits<KV>::to_float(kc[i]));
        vb[i] = __float2bfloat16_rn(KvTraits<KV>::to_float(vc[i]));
    }
}

// Cache rows from row0 up of layers [0, n) changed outside the shadows' writers: lower their marks.
__global__ void shadow_lower_kernel(int* wm, int n, int row0) {
    for (int l = threadIdx.x; l < n; l += blockDim.x) wm[l] = min(wm[l], row0);
}

}  // namespace lg
