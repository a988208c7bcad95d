/*
 * compactlogic_b200 — C ABI of the B200 (sm_100a) CompactLogic logic-layer hot path.
 *
 * Conventions
 *   - Every pointer argument is a device pointer unless its name ends in `_host`.
 *   - Every buffer is allocated by the caller.  No compute entry point allocates device memory;
 *     entry points that need temporary device memory take a caller-provided `workspace` and have a
 *     matching `*_workspace_bytes` query.  The one exception is clb_peer_alloc (width-sharded
 *     training), whose job is to cudaMalloc a buffer that other processes map over CUDA IPC.
 *   - `stream` is a cudaStream_t (pass the caller's current stream; 0 = legacy default stream).
 *     All work is enqueued asynchronously on it.  Entry points marked (sync) read a device flag
 *     back and so synchronise with the stream.
 *   - Return value: CLB_OK or a CLB_ERR_* code; clb_last_error() gives a message for the calling
 *     thread.  No entry point ever terminates the process (the reference aborts via exit() on a CUDA
 *     error, compactlogic/cuda/utils.cuh:46-53).
 *   - Activations are feature-major: x[feature][column] with row stride `ld` elements (the
 *     reference dense layout, compactlogic/cuda/difflogic_kernel.cu:8-12), unless stated otherwise.
 *
 * Two groups of entry points:
 *   1. clb_difflogic_* / clb_convlogic_* / clb_tensor_packbits / clb_groupbitsum mirror, one to one,
 *      the functions of the reference's pybind modules `difflogic_cuda` and `convlogic_cuda`
 *      (compactlogic/cuda/difflogic.cpp:60-105, compactlogic/cuda/convlogic.cpp:49-110), with the
 *      same tensor layouts, argument meaning and results.
 *   2. clb_logic_* / clb_slots_* / clb_packed_* are the native fast path used by the Python layers
 *      (softmax and its backward fused, int32 slot tables, fused GroupSum, bit-packed inference).
 */
#ifndef COMPACTLOGIC_B200_H
#define COMPACTLOGIC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* clb_stream_t; /* cudaStream_t */

enum clb_status {
    CLB_OK = 0,
    CLB_ERR_INVALID = 1,      /* bad shape / size / null pointer / unsupported option */
    CLB_ERR_DTYPE = 2,        /* unsupported element type */
    CLB_ERR_INDEX = 3,        /* a connection index or offset points outside the input */
    CLB_ERR_CUDA = 4,         /* a CUDA launch or runtime call failed */
    CLB_ERR_WORKSPACE = 5,    /* workspace too small */
    CLB_ERR_DIVISIBILITY = 6  /* groupbitsum: rows not divisible by k (reference raises ValueError) */
};

enum clb_dtype { CLB_F32 = 0, CLB_F64 = 1, CLB_BF16 = 2, CLB_F16 = 3 };  /* fp16 and bf16 compute in fp32 */

/* How a layer's per-row weights are interpreted. */
enum clb_weight_mode {
    CLB_W_LOGITS = 0, /* raw gate logits; softmax over K taken in-kernel (compactlogic.py:108) */
    CLB_W_PROBS = 1,  /* probabilities, as the reference kernels receive them */
    CLB_W_SELECT = 2  /* discrete: one chosen slot per row (`select`), gate output unweighted */
};

const char* clb_last_error(void);
int clb_abi_version(void);
/* Number of kernels this library launched since load (host-side counter, all threads). */
long long clb_launch_count(void);

/* ============================== 1. reference-mirroring entry points ==============================
 * Dtypes: as the reference — fp32 / fp64 / fp16 for the dense entry points
 * (AT_DISPATCH_FLOATING_TYPES_AND_HALF, difflogic_kernel.cu:222), fp32 / fp64 for conv.  fp16 computes in
 * fp32 and its fp32 copies of w / grad_y / results live in the workspace.  Indices a, b are int64
 * [out_dim, K] (the two halves of the layer's `indices` buffer), gate_seq uint8 [out_dim, K], w [out_dim, K]
 * and grad tensors in the activation dtype.
 */

/* Replaces difflogic_cuda.forward(x, a, b, w, gate_seq) -> y  (compactlogic/cuda/difflogic.cpp:61-66,
 * compactlogic/cuda/difflogic_kernel.cu:197-236).  x [in_dim, batch], y [out_dim, batch]. */
size_t clb_difflogic_workspace_bytes(int64_t in_dim, int64_t out_dim, int64_t K, int64_t batch, int dtype);
int clb_difflogic_forward(int dtype, const void* x, int64_t in_dim, int64_t batch, const int64_t* a,
                          const int64_t* b, const void* w, const uint8_t* gate_seq, int64_t out_dim, int64_t K,
                          void* y, void* workspace, size_t workspace_bytes, clb_stream_t stream);

/* Replaces difflogic_cuda.backward_w(x, a, b, gate_seq, grad_y) -> grad_w (d loss / d prob)
 * (compactlogic/cuda/difflogic.cpp:67-71, difflogic_kernel.cu:239-282).  grad_w [out_dim, K]. */
int clb_difflogic_backward_w(int dtype, const void* x, int64_t in_dim, int64_t batch, const int64_t* a,
                             const int64_t* b, const uint8_t* gate_seq, const void* grad_y, int64_t out_dim,
                             int64_t K, void* grad_w, void* workspace, size_t workspace_bytes, clb_stream_t stream);

/* No counterpart in the reference.  Same result as clb_difflogic_backward_w for fp32 and fp64 (fp16
 * returns CLB_ERR_DTYPE: its fp32 staging copies would not fit the fixed scratch), for callers that
 * cannot allocate device memory (no allocator of their own to provide a workspace, or an allocator
 * that forbids cudaMalloc where the call is made): instead of a workspace it uses an 8 MiB scratch
 * array compiled into the library, held on every GPU that loads it until exit.  Limit:
 *   round256(out_dim*K*8) + round256(chunks*out_dim*K*elem) <= 8 MiB,
 * chunks = clb_logic_backward_chunks(dtype, x, batch, batch, in_dim, grad_y, batch, NULL, 0, NULL, batch)
 * (the column split depends on the pointers' alignment and the tuning environment, so query it
 * rather than assume 128 columns per chunk), elem = 4 (fp32) or 8 (fp64); larger calls return
 * CLB_ERR_WORKSPACE.  The first call on a device (with it current) looks up the array's address
 * and caches it for the process's current context on that device (after cudaDeviceReset the cached
 * address is stale: do not call this entry point again in that process); make that first call
 * before any stream capture.  Calls share the array: calls that overlap on the GPU race and must be
 * serialised by the caller.  Allocates nothing. */
int clb_difflogic_backward_w_noalloc(int dtype, const void* x, int64_t in_dim, int64_t batch, const int64_t* a,
                                     const int64_t* b, const uint8_t* gate_seq, const void* grad_y, int64_t out_dim,
                                     int64_t K, void* grad_w, clb_stream_t stream);

/* Replaces difflogic_cuda.backward_x(x, a, b, w, gate_seq, grad_y, starts, ys, gate_codes) -> grad_x
 * (compactlogic/cuda/difflogic.cpp:72-77, difflogic_kernel.cu:285-333): a deterministic gather over
 * the inverse connection index built by LogicLayer.refresh_backward_index (compactlogic.py:184-274).
 * starts int64 [in_dim+1], ys int64 [2*out_dim*K], gate_codes int8 [2*out_dim*K]. */
int clb_difflogic_backward_x(int dtype, const void* x, int64_t in_dim, int64_t batch, const int64_t* a,
                             const int64_t* b, const void* w, const uint8_t* gate_seq, const void* grad_y,
                             const int64_t* starts, const int64_t* ys, const int8_t* gate_codes, int64_t out_dim,
                             int64_t K, void* grad_x, void* workspace, size_t workspace_bytes, clb_stream_t stream);

/* Replaces difflogic_cuda.backward_x_atomicAdd(x, a, b, w, gate_seq, grad_y) -> grad_x
 * (compactlogic/cuda/difflogic.cpp:99-104, difflogic_kernel.cu:613-656): scatter formulation.
 * Unlike the reference it does not synchronise the device. */
int clb_difflogic_backward_x_atomic(int dtype, const void* x, int64_t in_dim, int64_t batch, const int64_t* a,
                                    const int64_t* b, const void* w, const uint8_t* gate_seq, const void* grad_y,
                                    int64_t out_dim, int64_t K, void* grad_x, void* workspace,
                                    size_t workspace_bytes, clb_stream_t stream);

/* Replaces difflogic_cuda.eval(x, a, b, w_u8, gate_seq) -> y (compactlogic/cuda/difflogic.cpp:78-83,
 * difflogic_kernel.cu:341-411): the argmax gate's real polynomial, w_u8 [out_dim] selects the slot. */
int clb_difflogic_eval(int dtype, const void* x, int64_t in_dim, int64_t batch, const int64_t* a,
                       const int64_t* b, const uint8_t* w_sel, const uint8_t* gate_seq, int64_t out_dim, int64_t K,
                       void* y, void* workspace, size_t workspace_bytes, clb_stream_t stream);

/* Replaces difflogic_cuda.tensor_packbits_cuda(t, bit_count) -> (words, pad_len)
 * (compactlogic/cuda/difflogic.cpp:84-89, difflogic_kernel.cu:453-494).  t bool/uint8 [rows, cols];
 * out [rows, ceil(cols/bit_count)] words of bit_count in {8,16,32,64} (bit i of word c = column
 * c*bit_count+i).  *pad_len_host receives (bit_count - cols % bit_count) % bit_count. */
int clb_tensor_packbits(const uint8_t* t, int64_t rows, int64_t cols, int bit_count, void* out,
                        int64_t* pad_len_host, clb_stream_t stream);

/* Replaces difflogic_cuda.groupbitsum(words, pad_len, k) -> counts [batch, k] int32
 * (compactlogic/cuda/difflogic.cpp:90-98, difflogic_kernel.cu:535-568), batch = nwords*bits - pad_len.
 * Returns CLB_ERR_DIVISIBILITY when rows % k != 0 (the reference raises ValueError). */
int clb_groupbitsum(const void* words, int64_t rows, int64_t nwords, int bit_count, int64_t pad_len, int64_t k,
                    int32_t* counts, clb_stream_t stream);

/* Conv layer, NCHW activations.  offsets_ch int32, offsets_h/offsets_w int8, all [2, c_out, K]
 * (compactlogic.py:642-698); stride/pad/ks as passed by ConvLayerCudaFunction (compactlogic.py:847-867).
 * h_out = (h_in + 2 pad - ks) / stride + 1 (convlogic_kernel.cu:159-160). */
size_t clb_convlogic_workspace_bytes(int64_t n, int64_t c_in, int64_t h_in, int64_t w_in, int64_t c_out,
                                     int64_t h_out, int64_t w_out, int64_t K, int dtype);

/* Replaces convlogic_cuda.forward(x, och, oh, ow, w, gate_seq, stride, pad, ks) -> y
 * (compactlogic/cuda/convlogic.cpp:50-60, convlogic_kernel.cu:140-188). */
int clb_convlogic_forward(int dtype, const void* x, int64_t n, int64_t c_in, int64_t h_in, int64_t w_in,
                          const int32_t* offsets_ch, const int8_t* offsets_h, const int8_t* offsets_w,
                          const void* w, const uint8_t* gate_seq, int64_t c_out, int64_t K, int stride, int pad,
                          int ks, void* y, void* workspace, size_t workspace_bytes, clb_stream_t stream);

/* Replaces convlogic_cuda.backward_x(x, och, oh, ow, w, gate_seq, grad_y, stride, pad) -> grad_x
 * (compactlogic/cuda/convlogic.cpp:61-75, convlogic_kernel.cu:248-293).  h_out/w_out come from grad_y. */
int clb_convlogic_backward_x(int dtype, const void* x, int64_t n, int64_t c_in, int64_t h_in, int64_t w_in,
                             const int32_t* offsets_ch, const int8_t* offsets_h, const int8_t* offsets_w,
                             const void* w, const uint8_t* gate_seq, const void* grad_y, int64_t c_out,
                             int64_t h_out, int64_t w_out, int64_t K, int stride, int pad, void* grad_x,
                             void* workspace, size_t workspace_bytes, clb_stream_t stream);

/* Replaces convlogic_cuda.backward_w(x, och, oh, ow, gate_seq, grad_y, stride) -> grad_w
 * (compactlogic/cuda/convlogic.cpp:76-89, convlogic_kernel.cu:385-430). */
int clb_convlogic_backward_w(int dtype, const void* x, int64_t n, int64_t c_in, int64_t h_in, int64_t w_in,
                             const int32_t* offsets_ch, const int8_t* offsets_h, const int8_t* offsets_w,
                             const uint8_t* gate_seq, const void* grad_y, int64_t c_out, int64_t h_out,
                             int64_t w_out, int64_t K, int stride, void* grad_w, void* workspace,
                             size_t workspace_bytes, clb_stream_t stream);

/* Replaces convlogic_cuda.eval(x, och, oh, ow, w_u8, gate_seq, stride, pad, ks) -> y
 * (compactlogic/cuda/convlogic.cpp:90-104, convlogic_kernel.cu:479-530). */
int clb_convlogic_eval(int dtype, const void* x, int64_t n, int64_t c_in, int64_t h_in, int64_t w_in,
                       const int32_t* offsets_ch, const int8_t* offsets_h, const int8_t* offsets_w,
                       const uint8_t* w_sel, const uint8_t* gate_seq, int64_t c_out, int64_t K, int stride, int pad,
                       int ks, void* y, void* workspace, size_t workspace_bytes, clb_stream_t stream);

/* ===================================== 2. native fast path =====================================
 * A layer is a slot table: slots int32 [n_out, K, 2] holds the input feature ids (a, b) of every
 * candidate gate of every output neuron, -1 meaning the constant 0 (conv zero padding).  Weights and
 * gates are per parameter row r = j / group: [n_out/group, K] (dense: group 1; conv: group =
 * h_out*w_out).  Weights are in the arithmetic type (fp32, or fp64 for fp64 activations).
 */

/* Slot table of a dense LogicLayer from its int64 `indices` halves (compactlogic.py:160-182).
 * err: optional device int32, OR-ed with 1 when an index is out of [0, in_dim); such slots read 0. */
int clb_slots_dense(const int64_t* a, const int64_t* b, int64_t n_out, int64_t K, int64_t in_dim, int32_t* slots,
                    int32_t* err, clb_stream_t stream);

/* Slot table of a ConvLayer (compactlogic.py:642-698, offsets already shifted by -padding).
 * Neuron j = (c * h_out + oy) * w_out + ox; input feature = (ch * h_in + y) * w_in + x. */
int clb_slots_conv(const int32_t* offsets_ch, const int8_t* offsets_h, const int8_t* offsets_w, int64_t c_out,
                   int64_t K, int64_t c_in, int64_t h_in, int64_t w_in, int64_t h_out, int64_t w_out, int stride,
                   int32_t* slots, int32_t* err, clb_stream_t stream);

/* in_features = rows of x: with the column count it selects the column-chunk geometry (very wide inputs
 * use narrower chunks so a chunk's slab of x stays in L2). */
/* Forward of one layer over columns [0, ncols) (LogicLayer.forward_cuda + LogicLayerCudaFunction.forward,
 * compactlogic.py:83-118,483-486; eval with mode CLB_W_SELECT, compactlogic.py:120-130).
 * If gs_acc != NULL the layer's GroupSum (compactlogic.py:450-468) is fused: y is not written and
 * gs_acc [gs_k, ld_gs] (arithmetic type, pre-zeroed) accumulates sum over the neurons of each class,
 * class(j) = j / gs_size. */
int clb_logic_forward(int dtype, const void* x, int64_t ldx, int64_t ncols, int64_t in_features, const int32_t* slots,
                      int64_t n_out,
                      int64_t K, int64_t group, int weight_mode, const void* weights, const uint8_t* gates,
                      const uint8_t* select, int has_pad, void* y, int64_t ldy, void* gs_acc, int64_t gs_k,
                      int64_t gs_size, int64_t ld_gs, clb_stream_t stream);

/* Same as clb_logic_forward, with the per-neuron stage (softmax over the K logits, gates compacted into
 * two- and one-operand entries, scaled row offsets) computed once into `stage` (caller-allocated,
 * 256-byte aligned, clb_logic_forward_stage_bytes bytes) instead of by every CTA of every column chunk.
 * Native refinement of LogicLayer.forward_cuda (compactlogic.py:83-118) — the reference rebuilds nothing
 * per chunk because its forward kernel reads logits-derived probabilities prepared by PyTorch
 * (compactlogic.py:108).  stage == NULL behaves as clb_logic_forward; a smaller stage returns
 * CLB_ERR_WORKSPACE.  Calls sharing one stage buffer must not overlap on the GPU. */
size_t clb_logic_forward_stage_bytes(int dtype, int64_t n_out, int64_t K);
int clb_logic_forward_staged(int dtype, const void* x, int64_t ldx, int64_t ncols, int64_t in_features,
                             const int32_t* slots, int64_t n_out, int64_t K, int64_t group, int weight_mode,
                             const void* weights, const uint8_t* gates, const uint8_t* select, int has_pad, void* y,
                             int64_t ldy, void* gs_acc, int64_t gs_k, int64_t gs_size, int64_t ld_gs, void* stage,
                             size_t stage_bytes, clb_stream_t stream);

/* Number of column chunks of the backward pass = rows of the partials scratch [nchunks, n_out, K]. */
int64_t clb_logic_backward_chunks(int dtype, const void* x, int64_t ldx, int64_t ncols, int64_t in_features,
                                  const void* grad_y, int64_t ldgy, const void* gs_grad, int64_t ld_gs, const void* grad_x,
                                  int64_t ldgx);

/* Fused backward of one layer (LogicLayerCudaFunction.backward, compactlogic.py:488-508):
 *  - grad_x (optional, [in, ldgx] arithmetic type): activation gradient; zeroed first when zero_grad_x.
 *  - partials (optional, [nchunks, n_out, K]): per-chunk d loss / d prob, folded by
 *    clb_logic_grad_finalize.  partials_chunks must equal clb_logic_backward_chunks() for the same
 *    pointers and strides (the column split depends on their 16-byte alignment).
 * grad_y [n_out, ldgy] arithmetic type; or, with gs_grad != NULL, the fused GroupSum's backward:
 * grad_y[j, n] = gs_grad[class(j), n] * gs_scale. */
int clb_logic_backward(int dtype, const void* x, int64_t ldx, int64_t ncols, const int32_t* slots, int64_t n_out,
                       int64_t K, int64_t group, int weight_mode, const void* weights, const uint8_t* gates,
                       int has_pad, const void* grad_y, int64_t ldgy, const void* gs_grad, int64_t gs_k,
                       int64_t gs_size, int64_t ld_gs, double gs_scale, void* grad_x, int64_t ldgx, int zero_grad_x,
                       int64_t in_features, void* partials, int64_t partials_chunks, clb_stream_t stream);

/* partials -> per-row gradient [n_out/group, K] in the arithmetic type: w.r.t. the logits (softmax
 * backward fused) for CLB_W_LOGITS, w.r.t. the probabilities for CLB_W_PROBS. */
int clb_logic_grad_finalize(int dtype, const void* partials, int64_t nchunks, int64_t n_out, int64_t K,
                            int64_t group, int weight_mode, const void* weights, void* grad_w, clb_stream_t stream);

/* ---- receptive-field-staged conv layers (fp32) ----
 * Native fast path of ConvLayer (compactlogic.py:598-640 with conv_layer_cuda_forward / _backward_x /
 * _backward_w / eval, compactlogic/cuda/convlogic_kernel.cu:86-530) for layers whose every slot reads
 * one input channel per output channel (the default num_chn == 1 connections).  x [c_in*h_in*w_in, ldx]
 * and y / grad_y [c_out*h_out*w_out, ld] are feature-major; off_h / off_w are the layer's int8
 * offsets_h / offsets_w buffers [2, c_out, K] (already shifted by -pad, each in [-pad, ks-1-pad]);
 * order [c_out] lists the output channels grouped by the input channel they read and starts
 * [c_in+1] delimits the groups; max_group is the largest group.  ncols, ldx and every ld must be
 * multiples of 4 and the pointers 16-byte aligned; K a power of two <= 32.  err (optional, device int32) gets bit 1 set if a
 * staging wait gave up (the kernel then skips its tile instead of hanging). */
int64_t clb_conv_plane_parts(int64_t h_out, int64_t w_out, int stride, int ks, int64_t ncols);
int clb_conv_plane_forward(int dtype, const void* x, int64_t ldx, int64_t ncols, int64_t c_in, int64_t h_in,
                           int64_t w_in, int64_t c_out, int64_t h_out, int64_t w_out, int stride, int pad, int ks,
                           int64_t K, const int8_t* off_h, const int8_t* off_w, const int32_t* order,
                           const int32_t* starts, int64_t max_group, int weight_mode, const void* weights,
                           const uint8_t* gates, const uint8_t* select, void* y, int64_t ldy, int32_t* err,
                           clb_stream_t stream);
/* grad_x (optional) [c_in*h_in*w_in, ldgx], zeroed first when zero_grad_x; partials
 * [clb_conv_plane_parts(), c_out, K] of d loss / d prob, folded by clb_logic_grad_finalize with
 * n_out = c_out and group = 1.  K must be 4, 8 or 16. */
int clb_conv_plane_backward(int dtype, const void* x, int64_t ldx, int64_t ncols, int64_t c_in, int64_t h_in,
                            int64_t w_in, int64_t c_out, int64_t h_out, int64_t w_out, int stride, int pad, int ks,
                            int64_t K, const int8_t* off_h, const int8_t* off_w, const int32_t* order,
                            const int32_t* starts, int64_t max_group, int weight_mode, const void* weights,
                            const uint8_t* gates, const void* grad_y, int64_t ldgy, void* grad_x, int64_t ldgx,
                            int zero_grad_x, void* partials, int64_t nparts, int32_t* err, clb_stream_t stream);

/* Measurement helper, no reference counterpart: throughput probe of the soft kernels' access pattern
 * (512-byte row gathers at hashed rows, mode 0; plus as many 512-byte red.global.add.v4.f32 row
 * reductions, mode 1) over src / dst slabs of `rows` rows (a power of two); `ctas` CTAs of 256 threads, `iters` steps
 * per warp; sink is a device float the loads are kept live through.  The benchmark sizes the slabs
 * like one column chunk of a layer and reports the kernels' L2 traffic against it. */
int clb_l2_probe(int mode, const float* src, float* dst, int64_t rows, int iters, int ctas, float* sink,
                 clb_stream_t stream);

/* ---- gather-form backward (destination-sorted, no scatter reductions) ----
 * The same gradients as clb_logic_backward, walked by destination: a per-layer index lists for every
 * input feature the slot operands that read it (the role of the reference's inverse connection index,
 * LogicLayer.refresh_backward_index, compactlogic.py:184-274, consumed by logic_layer_cuda_backward_x,
 * difflogic_kernel.cu:140-194, here extended so the same pass also yields the d loss / d prob partials of
 * logic_layer_cuda_backward_w, difflogic_kernel.cu:82-137).  One warp per input row and column chunk
 * gathers, for each occurrence, the other operand and grad_y of the slot's neuron; grad_x is stored once
 * (not accumulated, not atomically), and its summation order is fixed for a given index.
 * For fp32 with 16-byte rows and element offsets below 2^31 each call first bakes every occurrence into a
 * 32-byte record (offsets, p-scaled coefficients, the owner's gate) stored in the index buffer, so the index
 * must not be shared by calls that overlap on the GPU.  Requires n_out * K <= 2^24. */

/* Bytes of a layer's occurrence index (-1 if the sizes are out of range). */
int64_t clb_logic_index_bytes(int64_t n_out, int64_t K, int64_t in_features);

/* Build the occurrence index from the slot table and gate ids (rebuild whenever either changes).
 * `index` is a caller-owned device buffer of clb_logic_index_bytes() bytes. */
int clb_logic_index_build(const int32_t* slots, int64_t n_out, int64_t K, int64_t group, const uint8_t* gates,
                          int64_t in_features, void* index, int64_t index_bytes, clb_stream_t stream);

/* Column chunks of clb_logic_backward_gather = rows of its partials scratch [nchunks, n_out, K]. */
int64_t clb_logic_backward_gather_chunks(int dtype, const void* x, int64_t ldx, int64_t ncols, const void* grad_y,
                                         int64_t ldgy, const void* gs_grad, int64_t ld_gs, const void* grad_x,
                                         int64_t ldgx);

/* Fused gather-form backward.  grad_x [in_features, ldgx] (arithmetic type) is written in full;
 * partials (optional) as for clb_logic_backward, folded by clb_logic_grad_finalize; probs is a scratch
 * [n_out/group, K] of the arithmetic type (the per-step softmax).  grad_y / GroupSum arguments as for
 * clb_logic_backward; weight_mode CLB_W_LOGITS or CLB_W_PROBS. */
int clb_logic_backward_gather(int dtype, const void* x, int64_t ldx, int64_t ncols, int64_t in_features, int64_t n_out,
                              int64_t K, int64_t group, int weight_mode, const void* weights, const void* index,
                              const void* grad_y, int64_t ldgy, const void* gs_grad, int64_t gs_k, int64_t gs_size,
                              int64_t ld_gs, double gs_scale, void* grad_x, int64_t ldgx, void* probs, void* partials,
                              int64_t partials_chunks, clb_stream_t stream);

/* ---- width-sharded (neuron-parallel) training, one process per GPU ----
 * Each of n_peers ranks owns a contiguous share of a dense layer's neurons and every rank holds the
 * full input activations.  The collectives are fused into the layer kernels over NVLink peer memory:
 *  - forward: the neuron share's output rows are stored to every rank's full activation buffer,
 *    y_peers[p] = rank p's buffer + (first owned neuron) * ldy (an all-gather in the epilogue);
 *  - backward: grad_y of the owned neurons is the sum over ranks of their partial grad_x buffers of
 *    the following layer, gy_peers[p] = rank p's partial + (first owned neuron) * ldgy (a
 *    reduce-scatter in the grad_y load); grad_x is this rank's partial for the previous layer.
 * The caller orders the ranks around each call (a barrier after it) so that no rank reads a buffer
 * before every writer has finished.  y_peers / gy_peers are HOST arrays of n_peers <= 8 device
 * pointers, all with the same address modulo 16; group is 1 (dense layers).  Otherwise as
 * clb_logic_forward / clb_logic_backward (partials_chunks from clb_logic_backward_chunks with
 * grad_y = gy_peers[0]).  The reference has no distributed code; these have no reference counterpart. */
int clb_logic_forward_peers(int dtype, const void* x, int64_t ldx, int64_t ncols, int64_t in_features,
                            const int32_t* slots, int64_t n_out, int64_t K, int weight_mode, const void* weights,
                            const uint8_t* gates, int has_pad, void* const* y_peers, int n_peers, int64_t ldy,
                            clb_stream_t stream);
int clb_logic_backward_peers(int dtype, const void* x, int64_t ldx, int64_t ncols, const int32_t* slots,
                             int64_t n_out, int64_t K, int weight_mode, const void* weights, const uint8_t* gates,
                             int has_pad, const void* const* gy_peers, int n_peers, int64_t ldgy, void* grad_x,
                             int64_t ldgx, int zero_grad_x, int64_t in_features, void* partials,
                             int64_t partials_chunks, clb_stream_t stream);

/* Buffers shared between the ranks' processes: a device allocation of its own (cudaMalloc on the
 * current device), its 64-byte IPC handle, and the mapping of another process's handle into this
 * one (peer access enabled on first use). */
#define CLB_IPC_HANDLE_BYTES 64
int clb_peer_alloc(size_t bytes, void** ptr);
int clb_peer_free(void* ptr);
int clb_ipc_export(const void* ptr, void* handle);
int clb_ipc_import(const void* handle, void** ptr);
int clb_ipc_close(void* ptr);

/* Layout helpers: dst[c, r] = src[r, c] for elem_bytes in {1,2,4,8}; fp32 <-> bf16 casts. */
int clb_transpose(int elem_bytes, const void* src, int64_t rows, int64_t cols, int64_t ld_src, void* dst,
                  int64_t ld_dst, clb_stream_t stream);
int clb_cast(int src_dtype, const void* src, int dst_dtype, void* dst, int64_t n, clb_stream_t stream);

/* ---- training hooks ---- */

/* One step of EntropyRowResampler's per-row monitor for one layer (compactlogic/compactlogic.py:1113-1150):
 * h = normalised entropy of softmax(logits[r]) (weights_entropy, compactlogic.py:370-385); first call
 * (first != 0): ema = h, counter = 0; later: ema = decay*ema + (1-decay)*h, counter = |h - ema_old| < eps ?
 * counter + 1 : 0, converged[r] = counter >= patience.  n_converged (device int, zero it first) receives
 * the number of converged rows.  logits fp32 [rows, K]; ema fp32 / counter int32 / converged uint8 [rows]. */
int clb_entropy_monitor(const float* logits, int64_t rows, int64_t K, float ema_decay, float eps, int patience,
                        int first, float* ema, int32_t* counter, uint8_t* converged, int32_t* n_converged,
                        clb_stream_t stream);

/* Row resampling of LogicLayer.resample_connections (compactlogic/compactlogic.py:282-368) for the rows with
 * picked[r] != 0, in place, from caller-drawn random tensors of full size (so the row counts never reach the
 * host): draw_logits fp32 (N(0,1)), draw_gates uint8 (gate ids in [0, 16)), draw_a / draw_b int64 (inputs in
 * [0, in_dim)), all [rows, K].  Weak rows (max prob < threshold_low) take new logits, gates and inputs in
 * every slot; strong rows (max prob > threshold_high) keep their first argmax slot with logit
 * log(p (K-1) / (1-p)) (p clamped to [1e-6, 1-1e-6]; log(9 (K-1)) without keep_strong_weights), zero the
 * other logits and give those slots new gates and inputs.  Gates change only with update_gate.  changed[r]
 * (uint8) marks weak or strong rows; exp_avg / exp_avg_sq (optional, fp32 [rows, K], the optimizer's Adam
 * moments) are zeroed on changed rows (compactlogic.py:1152-1180); counter (optional, int32 [rows]) is reset
 * on every picked row (compactlogic.py:1146).  logits fp32 [rows, K], gates uint8 [rows, K], idx_a / idx_b
 * the two int64 [rows, K] halves of `indices`; K <= 32. */
int clb_resample_rows(float* logits, uint8_t* gates, int64_t* idx_a, int64_t* idx_b, int64_t rows, int64_t K,
                      const uint8_t* picked, float threshold_high, float threshold_low, int keep_strong_weights,
                      int update_gate, const float* draw_logits, const uint8_t* draw_gates, const int64_t* draw_a,
                      const int64_t* draw_b, uint8_t* changed, float* exp_avg, float* exp_avg_sq, int32_t* counter,
                      clb_stream_t stream);

/* ---- bit-packed discrete inference (uint64 words, bit i of word w = sample 64 w + i) ---- */

/* x [batch, features] sample-major with values in {0,1} (bit = x > 0.5) -> out [features, ldw]. */
int clb_pack_inputs(int dtype, const void* x, int64_t batch, int64_t features, int64_t ldx, uint64_t* out,
                    int64_t ldw, clb_stream_t stream);

/* Raw inputs x [batch, features] (e.g. pixels in [0,1]) -> nthr*features packed features: feature
 * t*features + f is x[:, f] > (t+1)/(nthr+1), the reference's threshold binarisation
 * (experiments/experiment_script.py:92, threshold-major channel order), fused with the packing. */
int clb_pack_thresholds(int dtype, const void* x, int64_t batch, int64_t features, int64_t ldx, int nthr,
                        uint64_t* out, int64_t ldw, clb_stream_t stream);

/* Frozen layer tables: sel_ab int32 [n_out, 2], sel_gate uint8 [n_out] from the slot table and the
 * per-row chosen slot (the `w` buffer of a frozen layer, or argmax of the logits; compactlogic.py:120-130). */
int clb_packed_select(const int32_t* slots, const uint8_t* gates, const uint8_t* select, int64_t n_out, int64_t K,
                      int64_t group, int32_t* sel_ab, uint8_t* sel_gate, clb_stream_t stream);

/* One packed layer over word columns [0, nwords): y[j, w] = gate_j(x[a_j, w], x[b_j, w]). */
int clb_packed_layer(const uint64_t* x, int64_t ldx, int64_t nwords, const int32_t* sel_ab, const uint8_t* sel_gate,
                     int64_t n_out, uint64_t* y, int64_t ldy, clb_stream_t stream);

/* Last packed layer fused with GroupSum: counts[(sample0 + n) * k + class] += number of neurons of the
 * class whose output bit for sample n is 1 (n < nsamples; class(j) = j / class_size).  counts int32
 * [*, k], accumulated (zero it first).  With a workspace of clb_packed_count_workspace_bytes() bytes
 * the per-CTA totals go through the workspace and are summed by a second kernel (no atomics on
 * counts, deterministic); with workspace == NULL (or too small) they are added atomically. */
size_t clb_packed_count_workspace_bytes(int64_t k, int64_t class_size, int64_t nwords);
int clb_packed_layer_count(const uint64_t* x, int64_t ldx, int64_t nwords, const int32_t* sel_ab,
                           const uint8_t* sel_gate, int64_t n_out, int64_t k, int64_t class_size, int32_t* counts,
                           int64_t sample0, int64_t nsamples, void* workspace, size_t workspace_bytes,
                           clb_stream_t stream);

/* Packed GroupSum over stored words [rows, nwords] uint64: same accumulation as above. */
int clb_packed_count(const uint64_t* words, int64_t rows, int64_t nwords, int64_t k, int64_t class_size,
                     int32_t* counts, int64_t sample0, int64_t nsamples, clb_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* COMPACTLOGIC_B200_H */
