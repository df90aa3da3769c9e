// flash_tc.cuh - bf16 tensor-core (tcgen05) attention for causal prefill and BERT.
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

inline const char*& tc_error_slot() {
    static thread_local const char* msg = "";
    return msg;
}
inline const char* tc_last_error() { return tc_error_slot(); }

inline int launch_flash_tc(const TcArgs&, int, cudaStream_t, int, int) {
    tc_error_slot() = "tensor-core attention kernel not built in this version";
    return 1;
}

}  // namespace lg
