// common.cuh - device helpers shared by the attention kernels (sm_100a only).
//
// mbarrier / TMA (cp.async.bulk.tensor into this CTA only) wrappers, bounded waits that give up after
// a deadline on %globaltimer and report through an error word instead of hanging, KV element
// traits, warp reductions and the seeded synthetic generator.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace lg {

// Error word written by kernels (device int).  0 = ok.
enum : int { KERR_OK = 0, KERR_TIMEOUT_FULL = 1, KERR_TIMEOUT_EMPTY = 2, KERR_TIMEOUT_PEER = 3,
             KERR_TIMEOUT_MMA = 4 };

// Every in-kernel wait gives up this long after the kernel started (ns of %globaltimer).
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Waits for the phase with `parity` to complete.  Returns false when the deadline passed or
// `*abort` (shared flag raised by another warp that gave up) became non-zero.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint64_t deadline, volatile int* abort) {
    uint32_t spins = 0;
    while (!mbar_try_wait(bar, parity)) {
        if ((++spins & 63u) == 0u) {
            if (*abort) return false;
            if (globaltimer_ns() > deadline) return false;
        }
    }
    return true;
}

// 1-D bulk copy global -> this CTA's shared memory (no multicast), completion counted on `bar`.
// Both addresses 16-byte aligned, `bytes` a multiple of 16.
__device__ __forceinline__ void bulk_copy_g2s(void* smem_dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
                 "l"(src), "r"(bytes), "r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
                 : "memory");
}

// ---------------------------------------------------------------------------------- TMA
// 3-D tiled load global -> shared, completion counted on `bar`.  Destination is this CTA's own
// shared memory only.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ uint4 lds128(const void* p) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "r"(smem_u32(p)));
    return r;
}

// ---------------------------------------------------------------------------------- KV traits
template <typename T>
struct KvTraits;

template <>
struct KvTraits<float> {
    static constexpr int kElemsPer16B = 4;
    __device__ static __forceinline__ void unpack(const uint4& r, float* x) {
        x[0] = __uint_as_float(r.x);
        x[1] = __uint_as_float(r.y);
        x[2] = __uint_as_float(r.z);
        x[3] = __uint_as_float(r.w);
    }
    __device__ static __forceinline__ float from_float(float v) { return v; }
    __device__ static __forceinline__ float to_float(float v) { return v; }
};

template <>
struct KvTraits<__half> {
    static constexpr int kElemsPer16B = 8;
    __device__ static __forceinline__ void unpack(const uint4& r, float* x) {
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
            x[2 * i] = f.x;
            x[2 * i + 1] = f.y;
        }
    }
    __device__ static __forceinline__ __half from_float(float v) { return __float2half_rn(v); }
    __device__ static __forceinline__ float to_float(__half v) { return __half2float(v); }
};

template <>
struct KvTraits<__nv_bfloat16> {
    static constexpr int kElemsPer16B = 8;
    __device__ static __forceinline__ void unpack(const uint4& r, float* x) {
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            x[2 * i] = __uint_as_float(w[i] << 16);
            x[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
        }
    }
    __device__ static __forceinline__ __nv_bfloat16 from_float(float v) {
        return __float2bfloat16_rn(v);
    }
    __device__ static __forceinline__ float to_float(__nv_bfloat16 v) {
        return __bfloat162float(v);
    }
};

// ---------------------------------------------------------------------------------- warps
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ---------------------------------------------------------------------------------- synth
__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
__host__ __device__ __forceinline__ uint64_t synth_base(uint64_t seed, uint64_t stream) {
    return splitmix64(seed ^ (stream * 0xD1B54A32D192ED03ull));
}
constexpr double kSynthSd = 37837.227241611614;  // sd of the sum of four uniforms on {0..65535}

__device__ __forceinline__ float synth_value(uint64_t base, uint64_t idx, float mul, float add) {
    const uint64_t r = splitmix64(base + idx);
    const int s = static_cast<int>(r & 0xFFFFu) + static_cast<int>((r >> 16) & 0xFFFFu) +
                  static_cast<int>((r >> 32) & 0xFFFFu) + static_cast<int>(r >> 48) - 131070;
    return __fadd_rn(__fmul_rn(static_cast<float>(s), mul), add);
}

}  // namespace lg
