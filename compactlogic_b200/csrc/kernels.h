// Internal launcher declarations shared by the kernel translation units and the C-ABI layer.
// Every launcher validates nothing: the C-ABI functions in capi.cu check arguments first.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace clb {

constexpr int kMaxPeers = 8;

// Arguments of one soft / select logic-layer pass over feature-major activations.
//   x      [in_features, ldx] element type `dtype`; columns [0, ncols) are processed.
//   slots  [n_out, K] pairs (a, b) of input feature ids; -1 reads as the constant 0 (padding).
//   weights, gates are per parameter row r = j / group  ([n_out / group, K]); a dense layer has
//   group 1, a conv layer shares one row across all h_out*w_out positions of a channel.
struct LayerArgs {
    int dtype;             // CLB_F32 / CLB_F64 / CLB_BF16
    const void* x;
    int64_t ldx;
    int64_t ncols;
    const int32_t* slots;  // int2 per (j, k)
    int64_t n_out;
    int K;
    int64_t group;
    int mode;              // CLB_W_LOGITS / CLB_W_PROBS / CLB_W_SELECT
    const void* weights;   // arithmetic type (fp32, or fp64 for fp64 activations)
    const uint8_t* gates;
    const uint8_t* select; // CLB_W_SELECT only: chosen slot per row
    bool has_pad;          // slots may contain -1
    int64_t in_features;   // rows of x (0 = unknown); selects the column-chunk geometry
};

// Width-sharded training (each rank owns a contiguous share of the neurons): the number of ranks and
// one pointer per rank.  Forward stores row j of y to p[r] + j*ldy for every rank r (the activation
// all-gather, fused into the epilogue as NVLink stores); backward reads grad_y[j] as the sum over r of
// p[r][j*ldgy] (the gradient reduce-scatter, fused into the grad_y load as NVLink reads).  Passed as
// its own kernel argument: growing LayerArgs changes the register allocation of the single-GPU kernels.
struct PeerArgs {
    int n;
    void* p[kMaxPeers];
};

struct GroupSumArgs {
    void* acc;         // [k, ld] arithmetic type: forward accumulates sum_j y[j, col] per class
    const void* grad;  // [k, ld] arithmetic type: backward reads d loss / d class sum
    int64_t k;
    int64_t size;      // neurons per class (after the reference's zero padding of out to k * size)
    int64_t ld;
    double scale;      // backward: grad_y[j, col] = grad[class(j), col] * scale
};

// stage != null: the forward stage is baked once into that buffer (logic_forward_stage_bytes bytes)
// instead of being rebuilt by every CTA of every column chunk.
cudaError_t launch_logic_forward(const LayerArgs& a, void* y, int64_t ldy, const GroupSumArgs* gs,
                                 cudaStream_t s, const PeerArgs* peers = nullptr, void* stage = nullptr);
size_t logic_forward_stage_bytes(int dtype, int64_t n_out, int64_t K);

// Fused backward: reads x once per slot and produces both the per-chunk partial sums of
// d loss / d prob (when `partials` != null) and the scattered activation gradient (when gx != null,
// accumulated into a pre-zeroed buffer).
// `part_chunks` must equal logic_backward_chunks(...) for the same arguments (checked).
cudaError_t launch_logic_backward(const LayerArgs& a, const void* gy, int64_t ldgy, const GroupSumArgs* gs,
                                  void* gx, int64_t ldgx, void* partials, int64_t part_chunks, cudaStream_t s,
                                  const PeerArgs* peers = nullptr);
int64_t logic_backward_chunks(int dtype, int64_t ncols, int64_t ldx, const void* x, int64_t ldgy,
                              const void* gy, int64_t ld_gs, const void* gs_grad, int64_t ldgx, const void* gx,
                              int64_t in_features);

// partials [nchunks, n_out, K] -> per-row gradient [n_out / group, K]: w.r.t. the logits (softmax
// backward fused) for CLB_W_LOGITS, w.r.t. the probabilities for CLB_W_PROBS.  `out_dtype` is the
// element type of `out` (the arithmetic type, or the activation type for the reference API).
cudaError_t launch_grad_finalize(const LayerArgs& a, const void* partials, int64_t nchunks, void* out,
                                 int out_dtype, cudaStream_t s);

// Reference-formulation grad_x: gather over the inverse connection index (deterministic).
cudaError_t launch_backward_x_csr(const LayerArgs& a, const void* gy, int64_t ldgy, int64_t in_dim,
                                  const int64_t* starts, const int64_t* ys, const int8_t* codes, void* gx,
                                  int64_t ldgx, cudaStream_t s);

// Slot tables.
cudaError_t launch_slots_dense(const int64_t* a, const int64_t* b, int64_t n_out, int64_t K, int64_t in_dim,
                               int32_t* slots, int32_t* err, cudaStream_t s);
cudaError_t launch_slots_conv(const int32_t* och, const int8_t* oh, const int8_t* ow, int64_t c_out, int64_t K,
                              int64_t c_in, int64_t h_in, int64_t w_in, int64_t h_out, int64_t w_out, int stride,
                              int32_t* slots, int32_t* err, cudaStream_t s);

// Layout changes between the reference's NCHW / [batch, features] and feature-major storage.
cudaError_t launch_transpose(int elem_bytes, const void* src, int64_t rows, int64_t cols, int64_t ld_src, void* dst,
                             int64_t ld_dst, cudaStream_t s);
cudaError_t launch_cast(int src_dtype, const void* src, int dst_dtype, void* dst, int64_t n, cudaStream_t s);

// Bit-packed discrete inference.
cudaError_t launch_packbits(const uint8_t* t, int64_t rows, int64_t cols, int64_t ld_t, int bits, uint8_t* out,
                            int64_t row_bytes, cudaStream_t s);
cudaError_t launch_groupbitsum(const uint8_t* words, int64_t rows, int64_t row_bytes, int64_t samples, int64_t k,
                               int64_t class_size, int32_t* counts, bool accumulate, int64_t sample0,
                               cudaStream_t s);
cudaError_t launch_pack_inputs(int dtype, const void* x, int64_t batch, int64_t features, int64_t ldx,
                               uint64_t* out, int64_t ldw, cudaStream_t s);
cudaError_t launch_pack_thresholds(int dtype, const void* x, int64_t batch, int64_t features, int64_t ldx, int nthr,
                                   uint64_t* out, int64_t ldw, cudaStream_t s);
cudaError_t launch_packed_select(const int32_t* slots, const uint8_t* gates, const uint8_t* select, int64_t n_out,
                                 int K, int64_t group, int32_t* sel_ab, uint8_t* sel_gate, cudaStream_t s);
cudaError_t launch_packed_layer(const uint64_t* x, int64_t ldx, int64_t nwords, const int32_t* sel_ab,
                                const uint8_t* sel_gate, int64_t n_out, uint64_t* y, int64_t ldy, cudaStream_t s);
cudaError_t launch_packed_layer_count(const uint64_t* x, int64_t ldx, int64_t nwords, const int32_t* sel_ab,
                                      const uint8_t* sel_gate, int64_t n_out, int64_t k, int64_t class_size,
                                      int32_t* counts, int64_t sample0, int64_t nsamples, void* ws, size_t ws_bytes,
                                      cudaStream_t s);
size_t packed_count_workspace_bytes(int64_t k, int64_t class_size, int64_t nwords);

// Fused entropy / EMA / patience monitor of EntropyRowResampler (hooks.cu).
cudaError_t launch_entropy_monitor(const float* logits, int64_t rows, int K, float inv_log_k, float* ema,
                                   int32_t* counter, int first, float decay, float eps, int patience,
                                   uint8_t* converged, int32_t* n_converged, cudaStream_t s);

// Device row resampling of LogicLayer.resample_connections from pre-drawn random tensors (hooks.cu).
cudaError_t launch_resample_rows(float* logits, uint8_t* gates, int64_t* idx_a, int64_t* idx_b, int64_t rows, int K,
                                 const uint8_t* picked, float high, float low, int keep_strong, int update_gate,
                                 const float* d_logits, const uint8_t* d_gates, const int64_t* d_a,
                                 const int64_t* d_b, uint8_t* changed, float* m1, float* m2, int32_t* counter,
                                 cudaStream_t s);

// Error / launch bookkeeping of the C ABI (capi.cu), for entry points defined in other files.
int set_error(int code, const char* msg);
void count_launches(int n);

}  // namespace clb
