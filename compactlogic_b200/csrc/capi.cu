// C ABI of the CompactLogic B200 hot path: argument checking, workspace carving, launches.
// The declarations (with the reference function each one replaces) are in
// include/compactlogic_b200.h.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <cmath>
#include <string>

#include "common.cuh"
#include "kernels.h"

using namespace clb;

namespace {

thread_local std::string g_err;
std::atomic<long long> g_launches{0};

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

int cuda_status(cudaError_t e, const char* where, int kernels = 1) {
    if (e != cudaSuccess) return fail(CLB_ERR_CUDA, "%s: %s", where, cudaGetErrorString(e));
    g_launches += kernels;
    g_err.clear();
    return CLB_OK;
}

size_t esize(int dtype) { return dtype == CLB_F64 ? 8 : (dtype == CLB_BF16 || dtype == CLB_F16) ? 2 : 4; }
size_t acc_size(int dtype) { return dtype == CLB_F64 ? 8 : 4; }
bool dtype_ok(int dtype) { return dtype == CLB_F32 || dtype == CLB_F64 || dtype == CLB_BF16 || dtype == CLB_F16; }
bool ref_dtype_ok(int dtype) { return dtype == CLB_F32 || dtype == CLB_F64 || dtype == CLB_F16; }
bool ref_conv_dtype_ok(int dtype) { return dtype == CLB_F32 || dtype == CLB_F64; }
size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }
cudaStream_t S(clb_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// Bump allocator over a caller-provided workspace.
struct Carve {
    char* base;
    size_t cap, used = 0;
    void* take(size_t bytes) {
        void* p = base + used;
        used += align256(bytes);
        return used <= cap ? p : nullptr;
    }
};

LayerArgs layer(int dtype, const void* x, int64_t ldx, int64_t ncols, const int32_t* slots, int64_t n_out, int64_t K,
                int64_t group, int mode, const void* weights, const uint8_t* gates, const uint8_t* select,
                bool has_pad, int64_t in_features = 0) {
    LayerArgs a{};
    a.in_features = in_features;
    a.dtype = dtype;
    a.x = x;
    a.ldx = ldx;
    a.ncols = ncols;
    a.slots = slots;
    a.n_out = n_out;
    a.K = (int)K;
    a.group = group;
    a.mode = mode;
    a.weights = weights;
    a.gates = gates;
    a.select = select;
    a.has_pad = has_pad;
    return a;
}

int check_layer(int dtype, int64_t n_out, int64_t K, int64_t group, int mode, const void* weights,
                const uint8_t* gates, const uint8_t* select, const int32_t* slots, bool need_weights = true) {
    if (!dtype_ok(dtype)) return fail(CLB_ERR_DTYPE, "unsupported dtype %d", dtype);
    if (n_out < 0 || K < 1 || K > 256) return fail(CLB_ERR_INVALID, "invalid n_out=%lld or K=%lld (1..256)", (long long)n_out, (long long)K);
    if (group < 1 || n_out % group) return fail(CLB_ERR_INVALID, "group %lld must divide n_out %lld", (long long)group, (long long)n_out);
    if (mode != CLB_W_LOGITS && mode != CLB_W_PROBS && mode != CLB_W_SELECT) return fail(CLB_ERR_INVALID, "bad weight mode %d", mode);
    if (n_out > 0 && (!slots || !gates)) return fail(CLB_ERR_INVALID, "null slots/gates");
    if (n_out > 0 && mode == CLB_W_SELECT && !select) return fail(CLB_ERR_INVALID, "select mode needs `select`");
    if (n_out > 0 && mode != CLB_W_SELECT && !weights && need_weights) return fail(CLB_ERR_INVALID, "null weights");
    return CLB_OK;
}

}  // namespace

namespace clb {
int set_error(int code, const char* msg) { return fail(code, "%s", msg); }
void count_launches(int n) { g_launches += n; }
}  // namespace clb

extern "C" {

const char* clb_last_error(void) { return g_err.c_str(); }
int clb_abi_version(void) { return 1; }
long long clb_launch_count(void) { return g_launches.load(); }

// ----------------------------------------------------------------------------------------------
// native fast path
// ----------------------------------------------------------------------------------------------
int clb_slots_dense(const int64_t* a, const int64_t* b, int64_t n_out, int64_t K, int64_t in_dim, int32_t* slots,
                    int32_t* err, clb_stream_t stream) {
    if (n_out < 0 || K < 1 || in_dim < 0) return fail(CLB_ERR_INVALID, "slots_dense: bad sizes");
    if (n_out * K > 0 && (!a || !b || !slots)) return fail(CLB_ERR_INVALID, "slots_dense: null pointer");
    return cuda_status(launch_slots_dense(a, b, n_out, K, in_dim, slots, err, S(stream)), "slots_dense");
}

int clb_slots_conv(const int32_t* och, const int8_t* oh, const int8_t* ow, int64_t c_out, int64_t K, int64_t c_in,
                   int64_t h_in, int64_t w_in, int64_t h_out, int64_t w_out, int stride, int32_t* slots, int32_t* err,
                   clb_stream_t stream) {
    if (c_out < 0 || K < 1 || c_in < 1 || h_in < 1 || w_in < 1 || h_out < 0 || w_out < 0 || stride < 1)
        return fail(CLB_ERR_INVALID, "slots_conv: bad sizes");
    if (c_out * K > 0 && (!och || !oh || !ow || !slots)) return fail(CLB_ERR_INVALID, "slots_conv: null pointer");
    if (c_in * h_in * w_in > INT32_MAX) return fail(CLB_ERR_INVALID, "slots_conv: input too large for int32 ids");
    return cuda_status(launch_slots_conv(och, oh, ow, c_out, K, c_in, h_in, w_in, h_out, w_out, stride, slots, err,
                                         S(stream)),
                       "slots_conv");
}

int clb_logic_forward(int dtype, const void* x, int64_t ldx, int64_t ncols, int64_t in_features, const int32_t* slots,
                      int64_t n_out,
                      int64_t K, int64_t group, int weight_mode, const void* weights, const uint8_t* gates,
                      const uint8_t* select, int has_pad, void* y, int64_t ldy, void* gs_acc, int64_t gs_k,
                      int64_t gs_size, int64_t ld_gs, clb_stream_t stream) {
    return clb_logic_forward_staged(dtype, x, ldx, ncols, in_features, slots, n_out, K, group, weight_mode, weights,
                                    gates, select, has_pad, y, ldy, gs_acc, gs_k, gs_size, ld_gs, nullptr, 0, stream);
}

size_t clb_logic_forward_stage_bytes(int dtype, int64_t n_out, int64_t K) {
    if (n_out < 1 || K < 1) return 0;
    return logic_forward_stage_bytes(dtype, n_out, K);
}

int clb_logic_forward_staged(int dtype, const void* x, int64_t ldx, int64_t ncols, int64_t in_features,
                             const int32_t* slots, int64_t n_out, int64_t K, int64_t group, int weight_mode,
                             const void* weights, const uint8_t* gates, const uint8_t* select, int has_pad, void* y,
                             int64_t ldy, void* gs_acc, int64_t gs_k, int64_t gs_size, int64_t ld_gs, void* stage,
                             size_t stage_bytes, clb_stream_t stream) {
    int st = check_layer(dtype, n_out, K, group, weight_mode, weights, gates, select, slots);
    if (st) return st;
    if (ncols < 0 || ldx < ncols) return fail(CLB_ERR_INVALID, "forward: ldx %lld < ncols %lld", (long long)ldx, (long long)ncols);
    if (ncols == 0 || n_out == 0) return CLB_OK;
    if (!x) return fail(CLB_ERR_INVALID, "forward: null x");
    if (stage != nullptr) {
        const size_t need = logic_forward_stage_bytes(dtype, n_out, K);
        if (stage_bytes < need || (uintptr_t)stage % 256 != 0)
            return fail(CLB_ERR_WORKSPACE, "forward: stage of %zu bytes (256-aligned) needed, got %zu", need, stage_bytes);
    }
    GroupSumArgs gs{};
    if (gs_acc) {
        if (gs_k < 1 || gs_size < 1 || ld_gs < ncols || gs_k * gs_size < n_out)
            return fail(CLB_ERR_INVALID, "forward: bad GroupSum geometry");
        gs.acc = gs_acc;
        gs.k = gs_k;
        gs.size = gs_size;
        gs.ld = ld_gs;
    } else {
        if (!y || ldy < ncols) return fail(CLB_ERR_INVALID, "forward: null y or ldy < ncols");
    }
    const LayerArgs a = layer(dtype, x, ldx, ncols, slots, n_out, K, group, weight_mode, weights, gates, select, has_pad,
                              in_features);
    return cuda_status(launch_logic_forward(a, y, ldy, gs_acc ? &gs : nullptr, S(stream), nullptr, stage),
                       "logic_forward_staged");
}

int64_t clb_logic_backward_chunks(int dtype, const void* x, int64_t ldx, int64_t ncols, int64_t in_features,
                                  const void* grad_y, int64_t ldgy, const void* gs_grad, int64_t ld_gs, const void* grad_x,
                                  int64_t ldgx) {
    return logic_backward_chunks(dtype, ncols, ldx, x, grad_y ? ldgy : ncols, grad_y, gs_grad ? ld_gs : ncols, gs_grad,
                                 grad_x ? ldgx : ncols, grad_x, in_features);
}

int clb_logic_backward(int dtype, const void* x, int64_t ldx, int64_t ncols, const int32_t* slots, int64_t n_out,
                       int64_t K, int64_t group, int weight_mode, const void* weights, const uint8_t* gates,
                       int has_pad, const void* grad_y, int64_t ldgy, const void* gs_grad, int64_t gs_k,
                       int64_t gs_size, int64_t ld_gs, double gs_scale, void* grad_x, int64_t ldgx, int zero_grad_x,
                       int64_t in_features, void* partials, int64_t partials_chunks, clb_stream_t stream) {
    // probabilities are only needed for grad_x (and logits always, for the softmax)
    int st = check_layer(dtype, n_out, K, group, weight_mode, weights, gates, nullptr, slots,
                         grad_x != nullptr || weight_mode == CLB_W_LOGITS);
    if (st) return st;
    if (weight_mode == CLB_W_SELECT) return fail(CLB_ERR_INVALID, "backward: select mode has no gradient");
    if (ncols < 0 || ldx < ncols) return fail(CLB_ERR_INVALID, "backward: ldx < ncols");
    if (grad_x && (ldgx < ncols || in_features < 0)) return fail(CLB_ERR_INVALID, "backward: ldgx < ncols");
    if (grad_x && zero_grad_x) {
        cudaError_t e = cudaMemsetAsync(grad_x, 0, acc_size(dtype) * (size_t)in_features * (size_t)ldgx, S(stream));
        if (e != cudaSuccess) return cuda_status(e, "backward: memset grad_x", 0);
    }
    if (ncols == 0 || n_out == 0) return CLB_OK;
    if (!x) return fail(CLB_ERR_INVALID, "backward: null x");
    GroupSumArgs gs{};
    if (gs_grad) {
        if (gs_k < 1 || gs_size < 1 || ld_gs < ncols || gs_k * gs_size < n_out)
            return fail(CLB_ERR_INVALID, "backward: bad GroupSum geometry");
        gs.grad = gs_grad;
        gs.k = gs_k;
        gs.size = gs_size;
        gs.ld = ld_gs;
        gs.scale = gs_scale;
    } else if (!grad_y || ldgy < ncols) {
        return fail(CLB_ERR_INVALID, "backward: null grad_y or ldgy < ncols");
    }
    const LayerArgs a = layer(dtype, x, ldx, ncols, slots, n_out, K, group, weight_mode, weights, gates, nullptr,
                              has_pad, in_features);
    if (partials) {
        const int64_t need = clb_logic_backward_chunks(dtype, x, ldx, ncols, in_features, gs_grad ? nullptr : grad_y, ldgy,
                                                       gs_grad,
                                                       ld_gs, grad_x, ldgx);
        if (need != partials_chunks)
            return fail(CLB_ERR_INVALID, "backward: partials sized for %lld chunks, this call needs %lld",
                        (long long)partials_chunks, (long long)need);
    }
    return cuda_status(launch_logic_backward(a, gs_grad ? nullptr : grad_y, ldgy, gs_grad ? &gs : nullptr, grad_x, ldgx,
                                             partials, partials_chunks, S(stream)),
                       "logic_backward");
}

int clb_logic_grad_finalize(int dtype, const void* partials, int64_t nchunks, int64_t n_out, int64_t K,
                            int64_t group, int weight_mode, const void* weights, void* grad_w, clb_stream_t stream) {
    if (!dtype_ok(dtype)) return fail(CLB_ERR_DTYPE, "finalize: dtype");
    if (K < 1 || K > 256 || group < 1 || n_out < 0 || n_out % group || nchunks < 0)
        return fail(CLB_ERR_INVALID, "finalize: bad sizes");
    if (weight_mode != CLB_W_LOGITS && weight_mode != CLB_W_PROBS) return fail(CLB_ERR_INVALID, "finalize: mode");
    if (n_out == 0) return CLB_OK;
    if (!grad_w || (nchunks > 0 && !partials) || (weight_mode == CLB_W_LOGITS && !weights))
        return fail(CLB_ERR_INVALID, "finalize: null pointer");
    const LayerArgs a = layer(dtype, nullptr, 0, 0, nullptr, n_out, K, group, weight_mode, weights, nullptr, nullptr, false);
    return cuda_status(launch_grad_finalize(a, partials, nchunks, grad_w, dtype, S(stream)), "grad_finalize");
}

// ----------------------------------------------------------------------------------------------
// width-sharded training: peer-stored forward, peer-summed backward, IPC-registered buffers
// ----------------------------------------------------------------------------------------------
namespace {
int set_peers(PeerArgs& a, const void* const* peers, int n_peers, const char* what) {
    if (n_peers < 1 || n_peers > kMaxPeers || !peers)
        return fail(CLB_ERR_INVALID, "%s: n_peers %d outside 1..%d", what, n_peers, kMaxPeers);
    const uintptr_t mis = reinterpret_cast<uintptr_t>(peers[0]) & 15;
    for (int p = 0; p < n_peers; ++p) {
        if (!peers[p]) return fail(CLB_ERR_INVALID, "%s: null peer pointer %d", what, p);
        // every rank's buffer is addressed with one stride and one vector width
        if ((reinterpret_cast<uintptr_t>(peers[p]) & 15) != mis)
            return fail(CLB_ERR_INVALID, "%s: peer pointers differ in 16-byte alignment", what);
        a.p[p] = const_cast<void*>(peers[p]);
    }
    a.n = n_peers;
    return CLB_OK;
}
}  // namespace

int clb_logic_forward_peers(int dtype, const void* x, int64_t ldx, int64_t ncols, int64_t in_features,
                            const int32_t* slots, int64_t n_out, int64_t K, int weight_mode, const void* weights,
                            const uint8_t* gates, int has_pad, void* const* y_peers, int n_peers, int64_t ldy,
                            clb_stream_t stream) {
    int st = check_layer(dtype, n_out, K, 1, weight_mode, weights, gates, nullptr, slots);
    if (st) return st;
    if (weight_mode == CLB_W_SELECT) return fail(CLB_ERR_INVALID, "forward_peers: select mode not supported");
    if (ncols < 0 || ldx < ncols || ldy < ncols) return fail(CLB_ERR_INVALID, "forward_peers: ld < ncols");
    const LayerArgs a = layer(dtype, x, ldx, ncols, slots, n_out, K, 1, weight_mode, weights, gates, nullptr, has_pad,
                              in_features);
    PeerArgs pa{};
    if ((st = set_peers(pa, const_cast<const void* const*>(y_peers), n_peers, "forward_peers"))) return st;
    if (ncols == 0 || n_out == 0) return CLB_OK;
    if (!x) return fail(CLB_ERR_INVALID, "forward_peers: null x");
    return cuda_status(launch_logic_forward(a, y_peers[0], ldy, nullptr, S(stream), &pa), "logic_forward_peers");
}

int clb_logic_backward_peers(int dtype, const void* x, int64_t ldx, int64_t ncols, const int32_t* slots,
                             int64_t n_out, int64_t K, int weight_mode, const void* weights, const uint8_t* gates,
                             int has_pad, const void* const* gy_peers, int n_peers, int64_t ldgy, void* grad_x,
                             int64_t ldgx, int zero_grad_x, int64_t in_features, void* partials,
                             int64_t partials_chunks, clb_stream_t stream) {
    int st = check_layer(dtype, n_out, K, 1, weight_mode, weights, gates, nullptr, slots,
                         grad_x != nullptr || weight_mode == CLB_W_LOGITS);
    if (st) return st;
    if (weight_mode == CLB_W_SELECT) return fail(CLB_ERR_INVALID, "backward_peers: select mode has no gradient");
    if (ncols < 0 || ldx < ncols || ldgy < ncols) return fail(CLB_ERR_INVALID, "backward_peers: ld < ncols");
    if (grad_x && (ldgx < ncols || in_features < 0)) return fail(CLB_ERR_INVALID, "backward_peers: ldgx < ncols");
    const LayerArgs a = layer(dtype, x, ldx, ncols, slots, n_out, K, 1, weight_mode, weights, gates, nullptr, has_pad,
                              in_features);
    PeerArgs pa{};
    if ((st = set_peers(pa, gy_peers, n_peers, "backward_peers"))) return st;
    if (grad_x && zero_grad_x) {
        cudaError_t e = cudaMemsetAsync(grad_x, 0, acc_size(dtype) * (size_t)in_features * (size_t)ldgx, S(stream));
        if (e != cudaSuccess) return cuda_status(e, "backward_peers: memset grad_x", 0);
    }
    if (ncols == 0 || n_out == 0) return CLB_OK;
    if (!x) return fail(CLB_ERR_INVALID, "backward_peers: null x");
    if (partials) {
        const int64_t need = clb_logic_backward_chunks(dtype, x, ldx, ncols, in_features, gy_peers[0], ldgy, nullptr, 0,
                                                       grad_x, ldgx);
        if (need != partials_chunks)
            return fail(CLB_ERR_INVALID, "backward_peers: partials sized for %lld chunks, this call needs %lld",
                        (long long)partials_chunks, (long long)need);
    }
    return cuda_status(launch_logic_backward(a, gy_peers[0], ldgy, nullptr, grad_x, ldgx, partials, partials_chunks,
                                             S(stream), &pa),
                       "logic_backward_peers");
}

static_assert(sizeof(cudaIpcMemHandle_t) == CLB_IPC_HANDLE_BYTES, "IPC handle size");

int clb_peer_alloc(size_t bytes, void** ptr) {
    if (!ptr) return fail(CLB_ERR_INVALID, "peer_alloc: null ptr");
    *ptr = nullptr;
    return cuda_status(cudaMalloc(ptr, bytes ? bytes : 256), "peer_alloc", 0);
}

int clb_peer_free(void* ptr) { return ptr ? cuda_status(cudaFree(ptr), "peer_free", 0) : CLB_OK; }

int clb_ipc_export(const void* ptr, void* handle) {
    if (!ptr || !handle) return fail(CLB_ERR_INVALID, "ipc_export: null pointer");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
    if (e != cudaSuccess) return cuda_status(e, "ipc_export", 0);
    memcpy(handle, &h, sizeof(h));
    return CLB_OK;
}

int clb_ipc_import(const void* handle, void** ptr) {
    if (!ptr || !handle) return fail(CLB_ERR_INVALID, "ipc_import: null pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    *ptr = nullptr;
    return cuda_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "ipc_import", 0);
}

int clb_ipc_close(void* ptr) { return ptr ? cuda_status(cudaIpcCloseMemHandle(ptr), "ipc_close", 0) : CLB_OK; }

int clb_transpose(int elem_bytes, const void* src, int64_t rows, int64_t cols, int64_t ld_src, void* dst,
                  int64_t ld_dst, clb_stream_t stream) {
    if (rows < 0 || cols < 0 || ld_src < cols || ld_dst < rows) return fail(CLB_ERR_INVALID, "transpose: bad sizes");
    if (rows * cols > 0 && (!src || !dst)) return fail(CLB_ERR_INVALID, "transpose: null");
    return cuda_status(launch_transpose(elem_bytes, src, rows, cols, ld_src, dst, ld_dst, S(stream)), "transpose");
}

int clb_cast(int src_dtype, const void* src, int dst_dtype, void* dst, int64_t n, clb_stream_t stream) {
    if (n < 0 || (n > 0 && (!src || !dst))) return fail(CLB_ERR_INVALID, "cast: bad args");
    return cuda_status(launch_cast(src_dtype, src, dst_dtype, dst, n, S(stream)), "cast");
}

int clb_pack_inputs(int dtype, const void* x, int64_t batch, int64_t features, int64_t ldx, uint64_t* out, int64_t ldw,
                    clb_stream_t stream) {
    if (!dtype_ok(dtype)) return fail(CLB_ERR_DTYPE, "pack_inputs: dtype");
    if (batch < 0 || features < 0 || ldx < features || ldw < (batch + 63) / 64)
        return fail(CLB_ERR_INVALID, "pack_inputs: bad sizes");
    if (batch * features > 0 && (!x || !out)) return fail(CLB_ERR_INVALID, "pack_inputs: null");
    return cuda_status(launch_pack_inputs(dtype, x, batch, features, ldx, out, ldw, S(stream)), "pack_inputs");
}

int clb_entropy_monitor(const float* logits, int64_t rows, int64_t K, float ema_decay, float eps, int patience,
                        int first, float* ema, int32_t* counter, uint8_t* converged, int32_t* n_converged,
                        clb_stream_t stream) {
    if (rows < 0 || K < 1) return fail(CLB_ERR_INVALID, "entropy_monitor: bad sizes");
    if (rows > 0 && (!logits || !ema || !counter || !converged || !n_converged))
        return fail(CLB_ERR_INVALID, "entropy_monitor: null");
    const float inv_log_k = K > 1 ? (float)(1.0 / log((double)K)) : 0.f;
    return cuda_status(launch_entropy_monitor(logits, rows, (int)K, inv_log_k, ema, counter, first, ema_decay, eps,
                                              patience, converged, n_converged, S(stream)),
                       "entropy_monitor");
}

int clb_resample_rows(float* logits, uint8_t* gates, int64_t* idx_a, int64_t* idx_b, int64_t rows, int64_t K,
                      const uint8_t* picked, float threshold_high, float threshold_low, int keep_strong_weights,
                      int update_gate, const float* draw_logits, const uint8_t* draw_gates, const int64_t* draw_a,
                      const int64_t* draw_b, uint8_t* changed, float* exp_avg, float* exp_avg_sq, int32_t* counter,
                      clb_stream_t stream) {
    if (rows < 0 || K < 1 || K > 32) return fail(CLB_ERR_INVALID, "resample_rows: K must be in [1, 32]");
    if (rows > 0 && (!logits || !gates || !idx_a || !idx_b || !picked || !draw_logits || !draw_gates || !draw_a ||
                     !draw_b || !changed))
        return fail(CLB_ERR_INVALID, "resample_rows: null");
    return cuda_status(launch_resample_rows(logits, gates, idx_a, idx_b, rows, (int)K, picked, threshold_high,
                                            threshold_low, keep_strong_weights, update_gate, draw_logits, draw_gates,
                                            draw_a, draw_b, changed, exp_avg, exp_avg_sq, counter, S(stream)),
                       "resample_rows");
}

int clb_pack_thresholds(int dtype, const void* x, int64_t batch, int64_t features, int64_t ldx, int nthr,
                        uint64_t* out, int64_t ldw, clb_stream_t stream) {
    if (!dtype_ok(dtype)) return fail(CLB_ERR_DTYPE, "pack_thresholds: dtype");
    if (batch < 0 || features < 0 || ldx < features || nthr < 1 || nthr > 64 || ldw < (batch + 63) / 64)
        return fail(CLB_ERR_INVALID, "pack_thresholds: bad sizes");
    if (batch * features > 0 && (!x || !out)) return fail(CLB_ERR_INVALID, "pack_thresholds: null");
    return cuda_status(launch_pack_thresholds(dtype, x, batch, features, ldx, nthr, out, ldw, S(stream)),
                       "pack_thresholds");
}

int clb_packed_select(const int32_t* slots, const uint8_t* gates, const uint8_t* select, int64_t n_out, int64_t K,
                      int64_t group, int32_t* sel_ab, uint8_t* sel_gate, clb_stream_t stream) {
    if (n_out < 0 || K < 1 || K > 256 || group < 1 || n_out % group) return fail(CLB_ERR_INVALID, "packed_select: sizes");
    if (n_out > 0 && (!slots || !gates || !select || !sel_ab || !sel_gate))
        return fail(CLB_ERR_INVALID, "packed_select: null");
    return cuda_status(launch_packed_select(slots, gates, select, n_out, (int)K, group, sel_ab, sel_gate, S(stream)),
                       "packed_select");
}

int clb_packed_layer(const uint64_t* x, int64_t ldx, int64_t nwords, const int32_t* sel_ab, const uint8_t* sel_gate,
                     int64_t n_out, uint64_t* y, int64_t ldy, clb_stream_t stream) {
    if (nwords < 0 || n_out < 0 || ldx < nwords || ldy < nwords) return fail(CLB_ERR_INVALID, "packed_layer: sizes");
    if (nwords * n_out > 0 && (!x || !sel_ab || !sel_gate || !y)) return fail(CLB_ERR_INVALID, "packed_layer: null");
    return cuda_status(launch_packed_layer(x, ldx, nwords, sel_ab, sel_gate, n_out, y, ldy, S(stream)), "packed_layer");
}

size_t clb_packed_count_workspace_bytes(int64_t k, int64_t class_size, int64_t nwords) {
    if (k < 1 || class_size < 1 || nwords < 1) return 0;
    return packed_count_workspace_bytes(k, class_size, nwords);
}

int clb_packed_layer_count(const uint64_t* x, int64_t ldx, int64_t nwords, const int32_t* sel_ab,
                           const uint8_t* sel_gate, int64_t n_out, int64_t k, int64_t class_size, int32_t* counts,
                           int64_t sample0, int64_t nsamples, void* workspace, size_t workspace_bytes,
                           clb_stream_t stream) {
    if (nwords < 0 || n_out < 0 || ldx < nwords || k < 1 || class_size < 1 || sample0 < 0 || nsamples < 0 ||
        nsamples > 64 * nwords)
        return fail(CLB_ERR_INVALID, "packed_layer_count: sizes");
    if (nwords * n_out > 0 && (!x || !sel_ab || !sel_gate || !counts))
        return fail(CLB_ERR_INVALID, "packed_layer_count: null");
    const int kernels = workspace ? 2 : 1;
    return cuda_status(launch_packed_layer_count(x, ldx, nwords, sel_ab, sel_gate, n_out, k, class_size, counts, sample0,
                                                 nsamples, workspace, workspace_bytes, S(stream)),
                       "packed_layer_count", kernels);
}

int clb_packed_count(const uint64_t* words, int64_t rows, int64_t nwords, int64_t k, int64_t class_size,
                     int32_t* counts, int64_t sample0, int64_t nsamples, clb_stream_t stream) {
    if (rows < 0 || nwords < 0 || k < 1 || class_size < 1 || nsamples < 0 || nsamples > 64 * nwords)
        return fail(CLB_ERR_INVALID, "packed_count: sizes");
    if (rows * nwords > 0 && (!words || !counts)) return fail(CLB_ERR_INVALID, "packed_count: null");
    return cuda_status(launch_groupbitsum(reinterpret_cast<const uint8_t*>(words), rows, nwords * 8, nsamples, k,
                                          class_size, counts, true, sample0, S(stream)),
                       "packed_count");
}

// ----------------------------------------------------------------------------------------------
// reference-mirroring entry points
// ----------------------------------------------------------------------------------------------
size_t clb_difflogic_workspace_bytes(int64_t in_dim, int64_t out_dim, int64_t K, int64_t batch, int dtype) {
    const int64_t chunks = (batch + 31) / 32;  // upper bound (scalar path)
    size_t b = align256((size_t)out_dim * K * 8) + align256(4) + align256((size_t)chunks * out_dim * K * acc_size(dtype)) + 256;
    if (dtype == CLB_F16)  // fp32 copies of w, grad_y and of the result
        b += align256((size_t)out_dim * K * 4) + align256((size_t)out_dim * batch * 4) +
             align256((size_t)std::max(in_dim * batch, out_dim * K) * 4);
    return b;
}

namespace {
// fp16 entry points: fp32 staging of the probabilities, grad_y and the result in the workspace.
struct HalfStage {
    void* w = nullptr;
    void* gy = nullptr;
    void* out = nullptr;
};

int half_stage(int dtype, Carve& cv, int64_t in_dim, int64_t out_dim, int64_t K, int64_t batch, const void* w,
               const void* gy, HalfStage& h, cudaStream_t s) {
    if (dtype != CLB_F16) return CLB_OK;
    h.w = cv.take((size_t)out_dim * K * 4);
    h.gy = cv.take((size_t)out_dim * batch * 4);
    h.out = cv.take((size_t)std::max(in_dim * batch, out_dim * K) * 4);
    if (!h.out) return fail(CLB_ERR_WORKSPACE, "workspace too small for the fp16 staging");
    if (w) {
        cudaError_t e = launch_cast(CLB_F16, w, CLB_F32, h.w, out_dim * K, s);
        if (e != cudaSuccess) return cuda_status(e, "cast w");
    }
    if (gy) {
        cudaError_t e = launch_cast(CLB_F16, gy, CLB_F32, h.gy, out_dim * batch, s);
        if (e != cudaSuccess) return cuda_status(e, "cast grad_y");
    }
    return CLB_OK;
}
}  // namespace

static int dense_common(int dtype, const void* x, int64_t in_dim, int64_t batch, const int64_t* a, const int64_t* b,
                        int64_t out_dim, int64_t K, void* ws, size_t ws_bytes, Carve& cv, int32_t*& slots,
                        cudaStream_t s) {
    if (!ref_dtype_ok(dtype)) return fail(CLB_ERR_DTYPE, "reference dense API supports fp32/fp64/fp16 only");
    if (in_dim < 0 || batch < 0 || out_dim < 0 || K < 1 || K > 256) return fail(CLB_ERR_INVALID, "bad sizes");
    if ((in_dim * batch > 0 && !x) || (out_dim * K > 0 && (!a || !b))) return fail(CLB_ERR_INVALID, "null pointer");
    cv = Carve{reinterpret_cast<char*>(ws), ws_bytes};
    slots = reinterpret_cast<int32_t*>(cv.take((size_t)out_dim * K * 8));
    int32_t* err = reinterpret_cast<int32_t*>(cv.take(4));
    if (!ws || !slots || !err) return fail(CLB_ERR_WORKSPACE, "workspace too small (%zu bytes)", ws_bytes);
    return cuda_status(launch_slots_dense(a, b, out_dim, K, in_dim, slots, nullptr, s), "slots_dense");
}

int clb_difflogic_forward(int dtype, const void* x, int64_t in_dim, int64_t batch, const int64_t* a, const int64_t* b,
                          const void* w, const uint8_t* gate_seq, int64_t out_dim, int64_t K, void* y, void* workspace,
                          size_t workspace_bytes, clb_stream_t stream) {
    Carve cv{};
    int32_t* slots = nullptr;
    int st = dense_common(dtype, x, in_dim, batch, a, b, out_dim, K, workspace, workspace_bytes, cv, slots, S(stream));
    if (st) return st;
    HalfStage hs;
    if ((st = half_stage(dtype, cv, in_dim, out_dim, K, batch, w, nullptr, hs, S(stream)))) return st;
    if (dtype == CLB_F16) w = hs.w;
    return clb_logic_forward(dtype, x, batch, batch, in_dim, slots, out_dim, K, 1, CLB_W_PROBS, w, gate_seq, nullptr, 0, y,
                             batch, nullptr, 0, 0, 0, stream);
}

int clb_difflogic_eval(int dtype, const void* x, int64_t in_dim, int64_t batch, const int64_t* a, const int64_t* b,
                       const uint8_t* w_sel, const uint8_t* gate_seq, int64_t out_dim, int64_t K, void* y,
                       void* workspace, size_t workspace_bytes, clb_stream_t stream) {
    Carve cv{};
    int32_t* slots = nullptr;
    int st = dense_common(dtype, x, in_dim, batch, a, b, out_dim, K, workspace, workspace_bytes, cv, slots, S(stream));
    if (st) return st;
    return clb_logic_forward(dtype, x, batch, batch, in_dim, slots, out_dim, K, 1, CLB_W_SELECT, nullptr, gate_seq, w_sel, 0, y,
                             batch, nullptr, 0, 0, 0, stream);
}

int clb_difflogic_backward_w(int dtype, const void* x, int64_t in_dim, int64_t batch, const int64_t* a,
                             const int64_t* b, const uint8_t* gate_seq, const void* grad_y, int64_t out_dim, int64_t K,
                             void* grad_w, void* workspace, size_t workspace_bytes, clb_stream_t stream) {
    Carve cv{};
    int32_t* slots = nullptr;
    int st = dense_common(dtype, x, in_dim, batch, a, b, out_dim, K, workspace, workspace_bytes, cv, slots, S(stream));
    if (st) return st;
    HalfStage hs;
    if ((st = half_stage(dtype, cv, in_dim, out_dim, K, batch, nullptr, grad_y, hs, S(stream)))) return st;
    const void* gy = dtype == CLB_F16 ? hs.gy : grad_y;
    void* gw = dtype == CLB_F16 ? hs.out : grad_w;
    const int64_t chunks = clb_logic_backward_chunks(dtype, x, batch, batch, in_dim, gy, batch, nullptr, 0, nullptr, 0);
    void* part = cv.take((size_t)std::max<int64_t>(chunks, 1) * out_dim * K * acc_size(dtype));
    if (!part) return fail(CLB_ERR_WORKSPACE, "workspace too small for partials");
    // d loss / d prob does not depend on the probabilities: no weights needed
    st = clb_logic_backward(dtype, x, batch, batch, slots, out_dim, K, 1, CLB_W_PROBS, nullptr, gate_seq, 0, gy, batch,
                            nullptr, 0, 0, 0, 0.0, nullptr, 0, 0, in_dim, part, chunks, stream);
    if (st) return st;
    st = clb_logic_grad_finalize(dtype, part, batch > 0 ? chunks : 0, out_dim, K, 1, CLB_W_PROBS, nullptr, gw, stream);
    if (st || dtype != CLB_F16) return st;
    return cuda_status(launch_cast(CLB_F32, gw, CLB_F16, grad_w, out_dim * K, S(stream)), "cast grad_w");
}

int clb_difflogic_backward_x_atomic(int dtype, const void* x, int64_t in_dim, int64_t batch, const int64_t* a,
                                    const int64_t* b, const void* w, const uint8_t* gate_seq, const void* grad_y,
                                    int64_t out_dim, int64_t K, void* grad_x, void* workspace, size_t workspace_bytes,
                                    clb_stream_t stream) {
    Carve cv{};
    int32_t* slots = nullptr;
    int st = dense_common(dtype, x, in_dim, batch, a, b, out_dim, K, workspace, workspace_bytes, cv, slots, S(stream));
    if (st) return st;
    if (!grad_x && in_dim * batch > 0) return fail(CLB_ERR_INVALID, "null grad_x");
    HalfStage hs;
    if ((st = half_stage(dtype, cv, in_dim, out_dim, K, batch, w, grad_y, hs, S(stream)))) return st;
    const bool h = dtype == CLB_F16;
    st = clb_logic_backward(dtype, x, batch, batch, slots, out_dim, K, 1, CLB_W_PROBS, h ? hs.w : w, gate_seq, 0,
                            h ? hs.gy : grad_y, batch, nullptr, 0, 0, 0, 0.0, h ? hs.out : grad_x, batch, 1, in_dim,
                            nullptr, 0, stream);
    if (st || !h) return st;
    return cuda_status(launch_cast(CLB_F32, hs.out, CLB_F16, grad_x, in_dim * batch, S(stream)), "cast grad_x");
}

int clb_difflogic_backward_x(int dtype, const void* x, int64_t in_dim, int64_t batch, const int64_t* a,
                             const int64_t* b, const void* w, const uint8_t* gate_seq, const void* grad_y,
                             const int64_t* starts, const int64_t* ys, const int8_t* gate_codes, int64_t out_dim,
                             int64_t K, void* grad_x, void* workspace, size_t workspace_bytes, clb_stream_t stream) {
    Carve cv{};
    int32_t* slots = nullptr;
    int st = dense_common(dtype, x, in_dim, batch, a, b, out_dim, K, workspace, workspace_bytes, cv, slots, S(stream));
    if (st) return st;
    if (in_dim * batch == 0) return CLB_OK;
    if (!grad_x || !starts || (out_dim > 0 && (!ys || !gate_codes || !w || !gate_seq || !grad_y)))
        return fail(CLB_ERR_INVALID, "backward_x: null pointer");
    HalfStage hs;
    if ((st = half_stage(dtype, cv, in_dim, out_dim, K, batch, w, grad_y, hs, S(stream)))) return st;
    const bool h = dtype == CLB_F16;
    const LayerArgs la = layer(dtype, x, batch, batch, slots, out_dim, K, 1, CLB_W_PROBS, h ? hs.w : w, gate_seq, nullptr,
                               false);
    st = cuda_status(launch_backward_x_csr(la, h ? hs.gy : grad_y, batch, in_dim, starts, ys, gate_codes,
                                           h ? hs.out : grad_x, batch, S(stream)),
                     "backward_x_csr");
    if (st || !h) return st;
    return cuda_status(launch_cast(CLB_F32, hs.out, CLB_F16, grad_x, in_dim * batch, S(stream)), "cast grad_x");
}

int clb_tensor_packbits(const uint8_t* t, int64_t rows, int64_t cols, int bit_count, void* out, int64_t* pad_len_host,
                        clb_stream_t stream) {
    if (bit_count != 8 && bit_count != 16 && bit_count != 32 && bit_count != 64)
        return fail(CLB_ERR_INVALID, "`bit_count` has to be in { 8, 16, 32, 64 }");
    if (rows < 0 || cols < 0) return fail(CLB_ERR_INVALID, "packbits: bad sizes");
    const int64_t nwords = (cols + bit_count - 1) / bit_count;
    if (pad_len_host) *pad_len_host = (bit_count - cols % bit_count) % bit_count;
    if (rows * nwords == 0) return CLB_OK;
    if (!t || !out) return fail(CLB_ERR_INVALID, "packbits: null");
    return cuda_status(launch_packbits(t, rows, cols, cols, bit_count, reinterpret_cast<uint8_t*>(out),
                                       nwords * bit_count / 8, S(stream)),
                       "packbits");
}

int clb_groupbitsum(const void* words, int64_t rows, int64_t nwords, int bit_count, int64_t pad_len, int64_t k,
                    int32_t* counts, clb_stream_t stream) {
    if (bit_count != 8 && bit_count != 16 && bit_count != 32 && bit_count != 64)
        return fail(CLB_ERR_INVALID, "groupbitsum: word width must be 8, 16, 32 or 64 bits");
    if (k < 1 || rows < 0 || nwords < 0 || pad_len < 0 || pad_len > nwords * bit_count)
        return fail(CLB_ERR_INVALID, "groupbitsum: bad sizes");
    if (rows % k) {
        return fail(CLB_ERR_DIVISIBILITY, "in_dim (%lld) has to be divisible by k (%lld) but it is not", (long long)rows,
                    (long long)k);
    }
    const int64_t samples = nwords * bit_count - pad_len;
    if (samples == 0) return CLB_OK;
    if (!counts || (rows > 0 && !words)) return fail(CLB_ERR_INVALID, "groupbitsum: null");
    return cuda_status(launch_groupbitsum(reinterpret_cast<const uint8_t*>(words), rows, nwords * bit_count / 8, samples,
                                          k, rows / k, counts, false, 0, S(stream)),
                       "groupbitsum");
}

size_t clb_convlogic_workspace_bytes(int64_t n, int64_t c_in, int64_t h_in, int64_t w_in, int64_t c_out, int64_t h_out,
                                     int64_t w_out, int64_t K, int dtype) {
    const size_t e = esize(dtype);
    const size_t fin = (size_t)c_in * h_in * w_in, fout = (size_t)c_out * h_out * w_out;
    const size_t chunks = (size_t)(n + 31) / 32;
    return align256(fin * n * e) * 2 + align256(fout * K * 8) + align256(4) + align256(fout * n * e) * 2 +
           align256(chunks * fout * K * acc_size(dtype)) + 256;
}

namespace {
struct ConvWs {
    void* xT;
    void* gxT;
    int32_t* slots;
    void* yT;
    void* gyT;
    void* part;
};

int conv_common(int dtype, const void* x, int64_t n, int64_t c_in, int64_t h_in, int64_t w_in, const int32_t* och,
                const int8_t* oh, const int8_t* ow, int64_t c_out, int64_t h_out, int64_t w_out, int64_t K, int stride,
                void* ws, size_t ws_bytes, ConvWs& w, cudaStream_t s) {
    if (!ref_conv_dtype_ok(dtype)) return fail(CLB_ERR_DTYPE, "reference conv API supports fp32/fp64 only");
    if (n < 0 || c_in < 1 || h_in < 1 || w_in < 1 || c_out < 0 || h_out <= 0 || w_out <= 0 || K < 1 || K > 256 ||
        stride < 1)
        return fail(CLB_ERR_INVALID, "Invalid output shape: h_out=%lld, w_out=%lld", (long long)h_out, (long long)w_out);
    if ((n > 0 && !x) || (c_out > 0 && (!och || !oh || !ow))) return fail(CLB_ERR_INVALID, "conv: null pointer");
    const size_t e = esize(dtype);
    const size_t fin = (size_t)c_in * h_in * w_in, fout = (size_t)c_out * h_out * w_out;
    Carve cv{reinterpret_cast<char*>(ws), ws_bytes};
    w.xT = cv.take(fin * n * e);
    w.gxT = cv.take(fin * n * e);
    w.slots = reinterpret_cast<int32_t*>(cv.take(fout * K * 8));
    cv.take(4);
    w.yT = cv.take(fout * n * e);
    w.gyT = cv.take(fout * n * e);
    w.part = cv.take((size_t)((n + 31) / 32) * fout * K * acc_size(dtype));
    if (!ws || !w.part) return fail(CLB_ERR_WORKSPACE, "conv workspace too small (%zu bytes)", ws_bytes);
    int st = cuda_status(launch_slots_conv(och, oh, ow, c_out, K, c_in, h_in, w_in, h_out, w_out, stride, w.slots,
                                           nullptr, s),
                         "slots_conv");
    if (st) return st;
    return cuda_status(launch_transpose((int)e, x, n, (int64_t)fin, (int64_t)fin, w.xT, n, s), "transpose x");
}
}  // namespace

static int conv_forward_impl(int dtype, const void* x, int64_t n, int64_t c_in, int64_t h_in, int64_t w_in,
                             const int32_t* och, const int8_t* oh, const int8_t* ow, int mode, const void* w,
                             const uint8_t* sel, const uint8_t* gate_seq, int64_t c_out, int64_t K, int stride, int pad,
                             int ks, void* y, void* ws, size_t ws_bytes, clb_stream_t stream) {
    const int64_t h_out = (h_in + 2 * pad - ks) / stride + 1, w_out = (w_in + 2 * pad - ks) / stride + 1;
    ConvWs cw{};
    int st = conv_common(dtype, x, n, c_in, h_in, w_in, och, oh, ow, c_out, h_out, w_out, K, stride, ws, ws_bytes, cw,
                         S(stream));
    if (st) return st;
    const int64_t hw = h_out * w_out, fout = c_out * hw;
    if (n == 0 || fout == 0) return CLB_OK;
    st = clb_logic_forward(dtype, cw.xT, n, n, c_in * h_in * w_in, cw.slots, fout, K, hw, mode, w, gate_seq, sel, 1, cw.yT, n,
                           nullptr, 0, 0,
                           0, stream);
    if (st) return st;
    return cuda_status(launch_transpose((int)esize(dtype), cw.yT, fout, n, n, y, fout, S(stream)), "transpose y");
}

int clb_convlogic_forward(int dtype, const void* x, int64_t n, int64_t c_in, int64_t h_in, int64_t w_in,
                          const int32_t* offsets_ch, const int8_t* offsets_h, const int8_t* offsets_w, const void* w,
                          const uint8_t* gate_seq, int64_t c_out, int64_t K, int stride, int pad, int ks, void* y,
                          void* workspace, size_t workspace_bytes, clb_stream_t stream) {
    return conv_forward_impl(dtype, x, n, c_in, h_in, w_in, offsets_ch, offsets_h, offsets_w, CLB_W_PROBS, w, nullptr,
                             gate_seq, c_out, K, stride, pad, ks, y, workspace, workspace_bytes, stream);
}

int clb_convlogic_eval(int dtype, const void* x, int64_t n, int64_t c_in, int64_t h_in, int64_t w_in,
                       const int32_t* offsets_ch, const int8_t* offsets_h, const int8_t* offsets_w, const uint8_t* w_sel,
                       const uint8_t* gate_seq, int64_t c_out, int64_t K, int stride, int pad, int ks, void* y,
                       void* workspace, size_t workspace_bytes, clb_stream_t stream) {
    return conv_forward_impl(dtype, x, n, c_in, h_in, w_in, offsets_ch, offsets_h, offsets_w, CLB_W_SELECT, nullptr,
                             w_sel, gate_seq, c_out, K, stride, pad, ks, y, workspace, workspace_bytes, stream);
}

int clb_convlogic_backward_x(int dtype, const void* x, int64_t n, int64_t c_in, int64_t h_in, int64_t w_in,
                             const int32_t* offsets_ch, const int8_t* offsets_h, const int8_t* offsets_w, const void* w,
                             const uint8_t* gate_seq, const void* grad_y, int64_t c_out, int64_t h_out, int64_t w_out,
                             int64_t K, int stride, int pad, void* grad_x, void* workspace, size_t workspace_bytes,
                             clb_stream_t stream) {
    (void)pad;
    ConvWs cw{};
    int st = conv_common(dtype, x, n, c_in, h_in, w_in, offsets_ch, offsets_h, offsets_w, c_out, h_out, w_out, K,
                         stride, workspace, workspace_bytes, cw, S(stream));
    if (st) return st;
    const int64_t hw = h_out * w_out, fout = c_out * hw, fin = c_in * h_in * w_in;
    const size_t e = esize(dtype);
    if (n == 0) return CLB_OK;
    if (!grad_x || (fout > 0 && !grad_y)) return fail(CLB_ERR_INVALID, "conv backward_x: null");
    st = cuda_status(launch_transpose((int)e, grad_y, n, fout, fout, cw.gyT, n, S(stream)), "transpose grad_y");
    if (st) return st;
    st = clb_logic_backward(dtype, cw.xT, n, n, cw.slots, fout, K, hw, CLB_W_PROBS, w, gate_seq, 1, cw.gyT, n, nullptr,
                            0, 0, 0, 0.0, cw.gxT, n, 1, fin, nullptr, 0, stream);
    if (st) return st;
    return cuda_status(launch_transpose((int)e, cw.gxT, fin, n, n, grad_x, fin, S(stream)), "transpose grad_x");
}

int clb_convlogic_backward_w(int dtype, const void* x, int64_t n, int64_t c_in, int64_t h_in, int64_t w_in,
                             const int32_t* offsets_ch, const int8_t* offsets_h, const int8_t* offsets_w,
                             const uint8_t* gate_seq, const void* grad_y, int64_t c_out, int64_t h_out, int64_t w_out,
                             int64_t K, int stride, void* grad_w, void* workspace, size_t workspace_bytes,
                             clb_stream_t stream) {
    ConvWs cw{};
    int st = conv_common(dtype, x, n, c_in, h_in, w_in, offsets_ch, offsets_h, offsets_w, c_out, h_out, w_out, K,
                         stride, workspace, workspace_bytes, cw, S(stream));
    if (st) return st;
    const int64_t hw = h_out * w_out, fout = c_out * hw;
    const size_t e = esize(dtype);
    if (fout > 0 && n > 0) {
        if (!grad_y) return fail(CLB_ERR_INVALID, "conv backward_w: null grad_y");
        st = cuda_status(launch_transpose((int)e, grad_y, n, fout, fout, cw.gyT, n, S(stream)), "transpose grad_y");
        if (st) return st;
    }
    const int64_t chunks =
        n > 0 ? clb_logic_backward_chunks(dtype, cw.xT, n, n, c_in * h_in * w_in, cw.gyT, n, nullptr, 0, nullptr, 0) : 0;
    st = clb_logic_backward(dtype, cw.xT, n, n, cw.slots, fout, K, hw, CLB_W_PROBS, nullptr, gate_seq, 1, cw.gyT, n,
                            nullptr, 0, 0, 0, 0.0, nullptr, 0, 0, c_in * h_in * w_in, cw.part, chunks, stream);
    if (st) return st;
    return clb_logic_grad_finalize(dtype, cw.part, chunks, fout, K, hw, CLB_W_PROBS, nullptr, grad_w, stream);
}

}  // extern "C"
