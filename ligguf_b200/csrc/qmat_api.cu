// qmat_api.cu - the C ABI of the quantized projections (include/ligguf_cuda_attn.h, "quantized
// projections"): device-resident GGUF weight matrices, matmul / matmul2 / matmul3 on them for one
// token or a batch of prompt tokens, and the activation quantizers.  Nothing here falls back to the
// CPU.
#include <algorithm>
#include <cstring>
#include <numeric>
#include <vector>

#include "api_util.h"
#include "common.cuh"
#include "ligguf_cuda_attn.h"
#include "qmatvec.cuh"

using lgapi::DeviceGuard;
using lgapi::fail;

struct ligguf_qmat {
    int type = 0, n = 0, d = 0, device = 0, rb = 0;
    int ktype = 0;             // the kernel's layout of the rows: type, or QT_Q8_0_G32 when repacked
    uint8_t* w = nullptr;      // d rows of rb bytes, allocation padded to a 16-byte multiple
    int* h_err = nullptr;      // mapped pinned error word of the kernels that read this matrix
    int* d_err = nullptr;
    float* stage = nullptr;    // device staging of the host-pointer calls: x and the outputs
    size_t stage_floats = 0;
    uint8_t* act = nullptr;    // the activation forms of a call's token group (qmv_act_kernel)
    size_t act_bytes = 0;
    cudaStream_t stream = nullptr;
};

// A SARA reduce group member: this rank's buffer [2][nranks][rows] of 64-bit words, shared with the
// other ranks through CUDA IPC, and the device state of its epochs.
struct ligguf_reduce {
    int rows = 0, nranks = 0, rank = 0, device = 0;
    unsigned long long* buf = nullptr;
    unsigned long long** d_peers = nullptr;  // [nranks] buffer bases (own buffer for this rank)
    std::vector<void*> opened;
    int* d_state = nullptr;                  // [0] last completed epoch, [1] finished wait blocks
    int* h_err = nullptr;
    int* d_err = nullptr;
    bool open = false, pending = false;
};

namespace {

constexpr int kSmemLimit = 226 * 1024;
// Dynamic shared memory of one of two CTAs on an SM (228 KB per SM, 1 KB reserved per CTA and the
// kernel's few static bytes).
constexpr int kSmemHalf = 112 * 1024;

int row_bytes(int type, int n) {
    const int be = lg::qt_block_elems(type), bb = lg::qt_block_bytes(type);
    if (!be || n % be) return 0;
    return n / be * bb;
}

// Rows per ring stage: as many as fit kQmvStageMax, a multiple of the consumer warps when that many
// fit, and always a multiple of the rows that make the stage a whole number of 16-byte units (a
// bulk copy must start on a 16-byte boundary and move 16-byte multiples).
int tile_rows(int rb) {
    const int align = 16 / std::gcd(rb, 16);
    int r = lg::kQmvStageMax / rb;
    if (r >= lg::kQmvWarps) {
        const int step = std::lcm(align, lg::kQmvWarps);
        r = r / step * step;
        if (r == 0) r = lg::kQmvStageMax / rb / align * align;
    } else {
        r = r / align * align;
    }
    return r;
}

// Shared-memory layout of the activations of `tokens` tokens; returns their bytes.
int act_layout(lg::QmvArgs& a, int tokens) {
    auto up = [](int v, int m) { return (v + m - 1) / m * m; };
    int off = 0;
    lg::QmvAct& t = a.act;
    t = {};
    if (a.need_k) {
        t.off_qk = off;
        off = up(off + a.n, 16);
        t.off_dk = off;
        off = up(off + a.n / 256 * 4, 16);
        t.off_bs = off;
        off = up(off + a.n / 16 * 4, 16);
    }
    if (a.need_0) {
        t.off_q0 = off;
        off = up(off + a.n, 16);
        t.off_d0 = off;
        off = up(off + a.n / 32 * 4, 16);
    }
    if (a.need_f) {
        t.off_xf = off;
        off = up(off + a.n * 4, 16);
    }
    t.tok_bytes = off;
    t.bytes = up(off * tokens, 1024);
    return t.bytes;
}

// Ring stages next to `act` bytes of activations: the most (up to kQmvMaxStages) that let two CTAs
// share an SM; else the most that fit one CTA; 0 when not even two stages fit.
int ring_stages(int act) {
    for (int lim : {kSmemHalf, kSmemLimit})
        for (int s = lg::kQmvMaxStages; s >= 2; --s)
            if (act + s * lg::kQmvStageMax <= lim) return s;
    return 0;
}

int launch_act(const lg::QmvActArgs& qa, cudaStream_t st) {
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(std::max(1, (lg::qmv_act_items(qa) + 7) / 8), 1, 1);
    lc.blockDim = dim3(256, 1, 1);
    lc.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    LG_CUDA(cudaLaunchKernelEx(&lc, lg::qmv_act_kernel, qa));
    return LIGGUF_ATTN_OK;
}

template <int T>
int launch_qmv(lg::QmvArgs& a, int smem, int dev, cudaStream_t st) {
    auto kern = lg::qmv_kernel<T>;
    static int attr_bytes[64] = {};  // dynamic shared memory allowed so far on each device
    if (dev < 0 || dev >= 64 || attr_bytes[dev] < smem) {
        LG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        if (dev >= 0 && dev < 64) attr_bytes[dev] = smem;
    }
    int sms = 0;
    LG_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    cudaLaunchConfig_t lc = {};
    // Two CTAs per SM: the consumers are latency-bound, and 14 resident consumer warps per SM
    // measured 10-20 % faster than one CTA per SM with the next launch's CTA beside it.
    lc.gridDim = dim3(std::max(1, std::min(a.ntiles, 2 * sms)), 1, 1);
    lc.blockDim = dim3(lg::kQmvThreads, 1, 1);
    lc.dynamicSmemBytes = smem;
    lc.stream = st;
    // Programmatic dependent launch: the weights stream while the previous kernel finishes; the
    // consumers wait for it (griddepcontrol.wait) before reading x.
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    LG_CUDA(cudaLaunchKernelEx(&lc, kern, a));
    return LIGGUF_ATTN_OK;
}

// n_tok x rows of x (row stride x_stride) through up to three matrices; out_i row t at
// outs[i] + t * out_strides[i].  One launch per group of up to kQmvMaxTokens tokens (fewer when
// their activations would not fit shared memory next to the weight ring).
int matmul_enqueue(const ligguf_qmat* const* ws, float* const* outs, const long long* out_strides, int nmat,
                   const float* d_x, long long x_stride, int n_tok, cudaStream_t st,
                   const ligguf_reduce* red = nullptr) {
    // x is read in 16-byte vectors: rows must start on 16-byte boundaries.
    if (!d_x || (reinterpret_cast<uintptr_t>(d_x) & 15) || (n_tok > 1 && (x_stride & 3)))
        return fail(LIGGUF_ATTN_EINVAL, "x must be non-null, 16-byte aligned, with a row stride of a multiple of 4 floats");
    lg::QmvArgs a = {};
    if (red) {
        a.red.peers = red->d_peers;
        a.red.state = red->d_state;
        a.red.nranks = red->nranks;
        a.red.rank = red->rank;
    }
    a.n = ws[0]->n;
    a.err = ws[0]->d_err;
    int tiles = 0;
    for (int i = 0; i < nmat; ++i) {
        const ligguf_qmat* w = ws[i];
        if (w->n != a.n) return fail(LIGGUF_ATTN_EINVAL, "matrices of one call have different input widths");
        if (w->device != ws[0]->device) return fail(LIGGUF_ATTN_EINVAL, "matrices of one call are on different devices");
        if (!outs[i] && !red) return fail(LIGGUF_ATTN_EINVAL, "null output");
        lg::QmvMat& m = a.m[a.nmat++];
        m.w = w->w;
        m.out = outs[i];
        m.out_stride = out_strides[i];
        m.type = w->ktype;
        m.rows = w->d;
        m.rb = w->rb;
        m.tile_rows = tile_rows(w->rb);
        m.tile0 = tiles;
        m.ntiles = (w->d + m.tile_rows - 1) / m.tile_rows;
        tiles += m.ntiles;
        a.need_k |= lg::qt_uses_q8k(w->type);
        a.need_0 |= lg::qt_uses_q80(w->type);
        a.need_f |= lg::qt_uses_f32(w->type);
    }
    a.ntiles = tiles;
    int T = lg::kQmvMaxTokens;
    while (T > 1 && (T / 2 >= n_tok || !ring_stages(act_layout(a, T)))) T /= 2;
    const int act = act_layout(a, T);
    a.stages = ring_stages(act);
    if (!a.stages)
        return fail(LIGGUF_ATTN_EUNSUPPORTED, "input width %d needs %d bytes of shared memory with these types",
                    a.n, act + 2 * lg::kQmvStageMax);
    const int smem = act + a.stages * lg::kQmvStageMax;
    if (size_t(a.act.tok_bytes) * T > ws[0]->act_bytes)
        return fail(LIGGUF_ATTN_EUNSUPPORTED, "activation forms of %d tokens exceed the matrix's scratch", T);
    lg::QmvActArgs qa = {};
    qa.n = a.n;
    qa.need_k = a.need_k;
    qa.need_0 = a.need_0;
    qa.need_f = a.need_f;
    qa.act = a.act;
    qa.out = ws[0]->act;
    qa.x_stride = x_stride;
    a.act_g = ws[0]->act;
    const int dev = ws[0]->device;
    for (int t0 = 0; t0 < n_tok; t0 += T) {
        // The group's activation forms, then the projection (each a programmatic dependent of the
        // kernel before it: the activation kernel waits for x, the projection streams its weights
        // before waiting for the forms; the next group's activation kernel waits for this
        // projection, so the scratch is free).
        a.n_tok = std::min(T, n_tok - t0);
        if (T == 1) {  // one token: the projection kernel quantizes it itself
            a.act_g = nullptr;
            a.x = d_x + t0 * x_stride;
        } else {
            qa.x = d_x + t0 * x_stride;
            qa.n_tok = a.n_tok;
            if (int rc = launch_act(qa, st)) return rc;
        }
        for (int i = 0; i < nmat; ++i) a.m[i].out = outs[i] ? outs[i] + t0 * out_strides[i] : nullptr;
        int rc;
        switch (T) {
            case 8: rc = launch_qmv<8>(a, smem, dev, st); break;
            case 4: rc = launch_qmv<4>(a, smem, dev, st); break;
            case 2: rc = launch_qmv<2>(a, smem, dev, st); break;
            default: rc = launch_qmv<1>(a, smem, dev, st); break;
        }
        if (rc) return rc;
    }
    return LIGGUF_ATTN_OK;
}

int check_qmat_err(const ligguf_qmat* w) {
    if (w->h_err && *reinterpret_cast<volatile int*>(w->h_err)) {
        const int code = *w->h_err;
        *reinterpret_cast<volatile int*>(w->h_err) = 0;
        return fail(LIGGUF_ATTN_ETIMEDOUT, "a bounded in-kernel wait of the projection gave up (code %d)", code);
    }
    return LIGGUF_ATTN_OK;
}

int batch_args(const ligguf_qmat* w0, const ligguf_qmat* w1, const ligguf_qmat* w2, int n_tok) {
    if (!w0) return fail(LIGGUF_ATTN_EINVAL, "null w0");
    if (!w1 && w2) return fail(LIGGUF_ATTN_EINVAL, "w2 without w1");
    if (n_tok < 1) return fail(LIGGUF_ATTN_EINVAL, "n_tok %d", n_tok);
    return LIGGUF_ATTN_OK;
}

}  // namespace

extern "C" {

size_t ligguf_cuda_qmat_row_bytes(int type, int n) { return n > 0 ? size_t(row_bytes(type, n)) : 0; }

int ligguf_cuda_qmat_free(ligguf_qmat* w) {
    if (!w) return LIGGUF_ATTN_OK;
    DeviceGuard dg(w->device);
    if (w->stream) cudaStreamSynchronize(w->stream);
    if (w->w) cudaFree(w->w);
    if (w->stage) cudaFree(w->stage);
    if (w->act) cudaFree(w->act);
    if (w->h_err) cudaFreeHost(w->h_err);
    if (w->stream) cudaStreamDestroy(w->stream);
    delete w;
    return LIGGUF_ATTN_OK;
}

int ligguf_cuda_qmat_init(int type, int n, int d, const void* rows, int rows_on_device, int device,
                          ligguf_qmat** out) {
    return ligguf_cuda_qmat_init_cols(type, n, d, rows, 0, n, rows_on_device, device, out);
}

int ligguf_cuda_qmat_init_cols(int type, int n, int d, const void* rows, int col0, int ncols, int rows_on_device,
                               int device, ligguf_qmat** out) {
    if (!out || !rows) return fail(LIGGUF_ATTN_EINVAL, "null argument");
    const int be = lg::qt_block_elems(type);
    if (!be) return fail(LIGGUF_ATTN_EUNSUPPORTED, "weight type %d has no kernel", type);
    if (col0 < 0 || ncols < 1 || col0 + ncols > n || col0 % be || ncols % be)
        return fail(LIGGUF_ATTN_EINVAL, "columns [%d, %d) of %d are not whole blocks of %d", col0, col0 + ncols, n, be);
    const int src_rb = row_bytes(type, n);
    if (!src_rb) return fail(LIGGUF_ATTN_EINVAL, "width %d is not a whole number of blocks", n);
    const size_t src_off = size_t(col0 / be) * lg::qt_block_bytes(type);
    n = ncols;
    *out = nullptr;
    if (n < 1 || d < 1) return fail(LIGGUF_ATTN_EINVAL, "non-positive size %d x %d", d, n);
    if (!lg::qt_block_bytes(type)) return fail(LIGGUF_ATTN_EUNSUPPORTED, "weight type %d has no kernel", type);
    const int rb = row_bytes(type, n);
    if (!rb || n % 32) return fail(LIGGUF_ATTN_EINVAL, "width %d is not a whole number of units of 32 of type %d", n, type);
    if (lg::qt_uses_q8k(type) && n % 256) return fail(LIGGUF_ATTN_EINVAL, "K-quant width %d is not a multiple of 256", n);
    if (n > lg::kQmvMaxN) return fail(LIGGUF_ATTN_EUNSUPPORTED, "width %d beyond %d", n, lg::kQmvMaxN);
    const int tr = tile_rows(rb);
    if (tr < 1 || size_t(tr) * rb > size_t(lg::kQmvStageMax))
        return fail(LIGGUF_ATTN_EUNSUPPORTED, "rows of %d bytes do not fit a %d-byte stage", rb, lg::kQmvStageMax);
    int ndev = 0;
    LG_CUDA(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev) return fail(LIGGUF_ATTN_EINVAL, "device %d of %d", device, ndev);
    DeviceGuard dg(device);
    ligguf_qmat* w = new ligguf_qmat();
    w->type = type;
    w->n = n;
    w->d = d;
    w->rb = rb;
    w->device = device;
    const size_t bytes = size_t(d) * rb;
    const size_t alloc = (bytes + 15) / 16 * 16 + 16;
    // Scratch for the activation forms of a token group: room for every form at once (Q8_K, Q8_0 and
    // the fp32 copy, each padded to 16 bytes), whichever types the matrices of a call have.
    w->act_bytes = size_t(lg::kQmvMaxTokens) * ((n + n / 64 + n / 4 + 48) + (n + n / 8 + 32) + (4 * n + 16));
    // rows of the source are src_rb bytes apart; the kept columns start src_off bytes into each
    if (cudaMalloc(&w->w, alloc) != cudaSuccess || cudaMemset(w->w, 0, alloc) != cudaSuccess ||
        cudaMemcpy2D(w->w, rb, static_cast<const uint8_t*>(rows) + src_off, src_rb, rb, d,
                     rows_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaHostAlloc(&w->h_err, 64, cudaHostAllocMapped) != cudaSuccess ||
        cudaHostGetDevicePointer(reinterpret_cast<void**>(&w->d_err), w->h_err, 0) != cudaSuccess ||
        cudaMalloc(&w->act, w->act_bytes) != cudaSuccess ||
        cudaStreamCreateWithFlags(&w->stream, cudaStreamNonBlocking) != cudaSuccess) {
        (void)cudaGetLastError();
        ligguf_cuda_qmat_free(w);
        return fail(LIGGUF_ATTN_ENOMEM, "weight matrix of %zu bytes", bytes);
    }
    *w->h_err = 0;
    w->ktype = type;
    // Q8_0 rows of a multiple of 1024 elements: repacked into groups of 32 blocks (the values of the
    // 32 blocks, then their scales; same bytes), so the kernel reads each unit with aligned loads.
    if (type == lg::QT_Q8_0 && n % 1024 == 0 && bytes > 0) {
        uint8_t* tmp = nullptr;
        const size_t n_blocks = bytes / 34;
        bool ok = cudaMalloc(&tmp, bytes) == cudaSuccess &&
                  cudaMemcpyAsync(tmp, w->w, bytes, cudaMemcpyDeviceToDevice, w->stream) == cudaSuccess;
        if (ok) {
            lg::repack_q80_g32_kernel<<<unsigned((n_blocks + 255) / 256), 256, 0, w->stream>>>(tmp, w->w, n_blocks);
            ok = cudaGetLastError() == cudaSuccess && cudaStreamSynchronize(w->stream) == cudaSuccess;
        }
        if (tmp) cudaFree(tmp);
        if (!ok) {
            (void)cudaGetLastError();
            ligguf_cuda_qmat_free(w);
            return fail(LIGGUF_ATTN_ENOMEM, "repacking a Q8_0 matrix of %zu bytes", bytes);
        }
        w->ktype = lg::QT_Q8_0_G32;
    }
    *out = w;
    return LIGGUF_ATTN_OK;
}

int ligguf_cuda_matmul3_batch_async(const ligguf_qmat* w0, const ligguf_qmat* w1, const ligguf_qmat* w2,
                                    const float* d_x, int n_tok, float* d_out0, float* d_out1, float* d_out2,
                                    void* stream) {
    int rc = batch_args(w0, w1, w2, n_tok);
    if (rc) return rc;
    if (!d_x) return fail(LIGGUF_ATTN_EINVAL, "null x");
    const ligguf_qmat* ws[3] = {w0, w1, w2};
    float* outs[3] = {d_out0, d_out1, d_out2};
    const long long strides[3] = {w0->d, w1 ? w1->d : 0, w2 ? w2->d : 0};
    const int nmat = w2 ? 3 : (w1 ? 2 : 1);
    DeviceGuard dg(w0->device);
    return matmul_enqueue(ws, outs, strides, nmat, d_x, w0->n, n_tok, static_cast<cudaStream_t>(stream));
}

int ligguf_cuda_matmul3_async(const ligguf_qmat* w0, const ligguf_qmat* w1, const ligguf_qmat* w2, const float* d_x,
                              float* d_out0, float* d_out1, float* d_out2, void* stream) {
    return ligguf_cuda_matmul3_batch_async(w0, w1, w2, d_x, 1, d_out0, d_out1, d_out2, stream);
}

int ligguf_cuda_matmul3_batch(const ligguf_qmat* w0, const ligguf_qmat* w1, const ligguf_qmat* w2, const float* x,
                              int n_tok, float* out0, float* out1, float* out2) {
    int rc = batch_args(w0, w1, w2, n_tok);
    if (rc) return rc;
    if (!x || !out0 || (w1 && !out1) || (w2 && !out2)) return fail(LIGGUF_ATTN_EINVAL, "null argument");
    ligguf_qmat* s = const_cast<ligguf_qmat*>(w0);
    DeviceGuard dg(s->device);
    const size_t d0 = w0->d, d1 = w1 ? w1->d : 0, d2 = w2 ? w2->d : 0;
    const size_t need = size_t(n_tok) * (w0->n + d0 + d1 + d2);
    if (s->stage_floats < need) {
        if (s->stage) cudaFree(s->stage);
        s->stage = nullptr;
        s->stage_floats = 0;
        if (cudaMalloc(&s->stage, need * sizeof(float)) != cudaSuccess)
            return fail(LIGGUF_ATTN_ENOMEM, "staging of %zu floats", need);
        s->stage_floats = need;
    }
    float* dx = s->stage;
    float* o0 = dx + size_t(n_tok) * w0->n;
    float* o1 = o0 + size_t(n_tok) * d0;
    float* o2 = o1 + size_t(n_tok) * d1;
    LG_CUDA(cudaMemcpyAsync(dx, x, size_t(n_tok) * w0->n * sizeof(float), cudaMemcpyHostToDevice, s->stream));
    rc = ligguf_cuda_matmul3_batch_async(w0, w1, w2, dx, n_tok, o0, w1 ? o1 : nullptr, w2 ? o2 : nullptr, s->stream);
    if (rc) return rc;
    LG_CUDA(cudaMemcpyAsync(out0, o0, size_t(n_tok) * d0 * sizeof(float), cudaMemcpyDeviceToHost, s->stream));
    if (w1) LG_CUDA(cudaMemcpyAsync(out1, o1, size_t(n_tok) * d1 * sizeof(float), cudaMemcpyDeviceToHost, s->stream));
    if (w2) LG_CUDA(cudaMemcpyAsync(out2, o2, size_t(n_tok) * d2 * sizeof(float), cudaMemcpyDeviceToHost, s->stream));
    LG_CUDA(cudaStreamSynchronize(s->stream));
    return check_qmat_err(w0);
}

int ligguf_cuda_matmul3(const ligguf_qmat* w0, const ligguf_qmat* w1, const ligguf_qmat* w2, const float* x,
                        float* out0, float* out1, float* out2) {
    return ligguf_cuda_matmul3_batch(w0, w1, w2, x, 1, out0, out1, out2);
}

// ---------------------------------------------------------------------------- SARA reduce
int ligguf_cuda_reduce_free(ligguf_reduce* r) {
    if (!r) return LIGGUF_ATTN_OK;
    DeviceGuard dg(r->device);
    cudaDeviceSynchronize();
    for (void* p : r->opened)
        if (p) cudaIpcCloseMemHandle(p);
    if (r->buf) cudaFree(r->buf);
    if (r->d_peers) cudaFree(r->d_peers);
    if (r->d_state) cudaFree(r->d_state);
    if (r->h_err) cudaFreeHost(r->h_err);
    delete r;
    return LIGGUF_ATTN_OK;
}

int ligguf_cuda_reduce_init(int rows, int nranks, int rank, int device, ligguf_reduce** out) {
    if (!out) return fail(LIGGUF_ATTN_EINVAL, "null out");
    *out = nullptr;
    if (rows < 1 || nranks < 1 || rank < 0 || rank >= nranks)
        return fail(LIGGUF_ATTN_EINVAL, "rows %d, rank %d of %d", rows, rank, nranks);
    int ndev = 0;
    LG_CUDA(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev) return fail(LIGGUF_ATTN_EINVAL, "device %d of %d", device, ndev);
    DeviceGuard dg(device);
    ligguf_reduce* r = new ligguf_reduce();
    r->rows = rows;
    r->nranks = nranks;
    r->rank = rank;
    r->device = device;
    const size_t words = 2 * size_t(nranks) * rows;
    if (cudaMalloc(&r->buf, words * 8) != cudaSuccess || cudaMemset(r->buf, 0, words * 8) != cudaSuccess ||
        cudaMalloc(&r->d_peers, nranks * sizeof(void*)) != cudaSuccess ||
        cudaMalloc(&r->d_state, 2 * sizeof(int)) != cudaSuccess ||
        cudaMemset(r->d_state, 0, 2 * sizeof(int)) != cudaSuccess ||
        cudaHostAlloc(&r->h_err, 64, cudaHostAllocMapped) != cudaSuccess ||
        cudaHostGetDevicePointer(reinterpret_cast<void**>(&r->d_err), r->h_err, 0) != cudaSuccess) {
        (void)cudaGetLastError();
        ligguf_cuda_reduce_free(r);
        return fail(LIGGUF_ATTN_ENOMEM, "reduce buffers");
    }
    *r->h_err = 0;
    *out = r;
    return LIGGUF_ATTN_OK;
}

int ligguf_cuda_reduce_ipc_handle(ligguf_reduce* r, void* handle_out, size_t handle_size) {
    if (!r || !handle_out) return fail(LIGGUF_ATTN_EINVAL, "null argument");
    if (handle_size < sizeof(cudaIpcMemHandle_t)) return fail(LIGGUF_ATTN_EINVAL, "handle buffer of %zu bytes", handle_size);
    DeviceGuard dg(r->device);
    cudaIpcMemHandle_t hd;
    LG_CUDA(cudaIpcGetMemHandle(&hd, r->buf));
    memcpy(handle_out, &hd, sizeof(hd));
    return LIGGUF_ATTN_OK;
}

int ligguf_cuda_reduce_open(ligguf_reduce* r, const void* handles, size_t handle_size) {
    if (!r || !handles) return fail(LIGGUF_ATTN_EINVAL, "null argument");
    if (handle_size < sizeof(cudaIpcMemHandle_t)) return fail(LIGGUF_ATTN_EINVAL, "handle stride %zu", handle_size);
    if (r->open) return fail(LIGGUF_ATTN_ESTATE, "reduce already open");
    DeviceGuard dg(r->device);
    std::vector<unsigned long long*> bases(r->nranks);
    r->opened.assign(r->nranks, nullptr);
    for (int p = 0; p < r->nranks; ++p) {
        if (p == r->rank) {
            bases[p] = r->buf;
            continue;
        }
        cudaIpcMemHandle_t hd;
        memcpy(&hd, static_cast<const char*>(handles) + size_t(p) * handle_size, sizeof(hd));
        void* ptr = nullptr;
        LG_CUDA(cudaIpcOpenMemHandle(&ptr, hd, cudaIpcMemLazyEnablePeerAccess));
        r->opened[p] = ptr;
        bases[p] = static_cast<unsigned long long*>(ptr);
    }
    LG_CUDA(cudaMemcpy(r->d_peers, bases.data(), bases.size() * sizeof(void*), cudaMemcpyHostToDevice));
    r->open = true;
    return LIGGUF_ATTN_OK;
}

int ligguf_cuda_matmul_reduce_async(const ligguf_qmat* w, ligguf_reduce* r, const float* d_x, void* stream) {
    if (!w || !r || !d_x) return fail(LIGGUF_ATTN_EINVAL, "null argument");
    if (!r->open) return fail(LIGGUF_ATTN_ESTATE, "reduce not open");
    if (r->pending) return fail(LIGGUF_ATTN_ESTATE, "the previous reduced projection has no reduce wait yet");
    if (w->d != r->rows) return fail(LIGGUF_ATTN_EINVAL, "matrix of %d rows into a reduce of %d", w->d, r->rows);
    if (w->device != r->device) return fail(LIGGUF_ATTN_EINVAL, "matrix and reduce on different devices");
    DeviceGuard dg(w->device);
    const ligguf_qmat* ws[1] = {w};
    float* outs[1] = {nullptr};
    const long long strides[1] = {0};
    const int rc = matmul_enqueue(ws, outs, strides, 1, d_x, w->n, 1, static_cast<cudaStream_t>(stream), r);
    if (!rc) r->pending = true;
    return rc;
}

int ligguf_cuda_reduce_wait_async(ligguf_reduce* r, float* d_x_inout, float* d_out, void* stream) {
    if (!r) return fail(LIGGUF_ATTN_EINVAL, "null argument");
    if (!r->open || !r->pending) return fail(LIGGUF_ATTN_ESTATE, "no reduced projection in flight");
    DeviceGuard dg(r->device);
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((r->rows + 255) / 256, 1, 1);
    lc.blockDim = dim3(256, 1, 1);
    lc.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    LG_CUDA(cudaLaunchKernelEx(&lc, lg::reduce_wait_kernel, static_cast<const unsigned long long*>(r->buf), r->d_state,
                               r->nranks, r->rows, d_x_inout, d_out, r->d_err));
    r->pending = false;
    return LIGGUF_ATTN_OK;
}

int ligguf_cuda_reduce_status(ligguf_reduce* r, void* stream) {
    if (!r) return fail(LIGGUF_ATTN_EINVAL, "null argument");
    DeviceGuard dg(r->device);
    LG_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
    if (*reinterpret_cast<volatile int*>(r->h_err)) {
        const int code = *r->h_err;
        *reinterpret_cast<volatile int*>(r->h_err) = 0;
        return fail(LIGGUF_ATTN_ETIMEDOUT, "a bounded wait of the reduce gave up (code %d)", code);
    }
    return LIGGUF_ATTN_OK;
}

int ligguf_cuda_quantize_q8_K_async(const float* d_x, int n, void* d_blocks, void* stream) {
    if (!d_x || !d_blocks) return fail(LIGGUF_ATTN_EINVAL, "null argument");
    if (n < 256 || n % 256) return fail(LIGGUF_ATTN_EINVAL, "n = %d is not a positive multiple of 256", n);
    const int nb = n / 256;
    lg::quantize_q8k_kernel<<<(nb + 7) / 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        d_x, nb, static_cast<uint8_t*>(d_blocks));
    LG_CUDA(cudaGetLastError());
    return LIGGUF_ATTN_OK;
}

int ligguf_cuda_quantize_q8_0_async(const float* d_x, int n, void* d_blocks, void* stream) {
    if (!d_x || !d_blocks) return fail(LIGGUF_ATTN_EINVAL, "null argument");
    if (n < 32 || n % 32) return fail(LIGGUF_ATTN_EINVAL, "n = %d is not a positive multiple of 32", n);
    const int nb = n / 32;
    lg::quantize_q80_kernel<<<(nb + 7) / 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        d_x, nb, static_cast<uint8_t*>(d_blocks));
    LG_CUDA(cudaGetLastError());
    return LIGGUF_ATTN_OK;
}

}  // extern "C"
