// Allocation-free variant of the reference backward_w entry point.
//
// Some callers of this library cannot allocate device memory at the point where they need the
// gate-probability gradient: code running under an allocator that forbids cudaMalloc (a host
// framework with a fixed arena, a caller inside a region where allocation would synchronise the
// device, or a plain C/FFI caller with no allocator of its own to hand out a workspace).
// clb_difflogic_backward_w needs a caller-provided workspace for its slot table and per-chunk
// partial sums; this variant instead uses a fixed scratch array compiled into the library.
//
// The scratch is a file-scope __device__ array of kNoAllocScratchBytes (8 MiB).  Every GPU that
// loads the library holds it until the process exits.  Host code cannot use the array's name as a
// device address (on the host it is only a stand-in symbol), so the first call on each device, with
// that device current, looks up the real address with cudaGetSymbolAddress and caches it; that
// first call should therefore happen before any stream capture.
//
// All calls share the one array: the slot table and the partial sums are fully rewritten by every
// call (nothing in it has to start at zero), but calls whose work overlaps on the GPU (different
// streams, or different host threads on the same device) race on it and must be serialised by the
// caller.
#include <cuda_runtime.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
constexpr int kMaxDevices = 128;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once per device).
int scratch_address(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return clb::set_error(CLB_ERR_CUDA, cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return clb::set_error(CLB_ERR_INVALID, "device index out of range");
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (g_scratch_addr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return clb::set_error(CLB_ERR_CUDA, cudaGetErrorString(e));
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return CLB_OK;
}

size_t round256(size_t v) { return (v + 255) & ~size_t(255); }

}  // namespace

extern "C" int clb_difflogic_backward_w_noalloc(int dtype, const void* x, int64_t in_dim, int64_t batch,
                                                const int64_t* a, const int64_t* b, const uint8_t* gate_seq,
                                                const void* grad_y, int64_t out_dim, int64_t K, void* grad_w,
                                                clb_stream_t stream) {
    if (dtype != CLB_F32 && dtype != CLB_F64) return clb::set_error(CLB_ERR_DTYPE, "fp32/fp64 only");
    if (in_dim < 0 || batch < 0 || out_dim < 0 || K < 1 || K > 256) return clb::set_error(CLB_ERR_INVALID, "bad sizes");
    if (out_dim == 0) return CLB_OK;
    if (!a || !b || !gate_seq || !grad_w || (batch > 0 && (!x || !grad_y)))
        return clb::set_error(CLB_ERR_INVALID, "null pointer");
    const size_t acc = dtype == CLB_F64 ? 8 : 4;
    const int64_t chunks =
        batch > 0 ? clb::logic_backward_chunks(dtype, batch, batch, x, batch, grad_y, 0, nullptr, batch, nullptr, in_dim)
                  : 0;
    const size_t slot_bytes = round256((size_t)out_dim * K * 8);
    const size_t need = slot_bytes + round256((size_t)chunks * out_dim * K * acc);
    if (need > kNoAllocScratchBytes)
        return clb::set_error(CLB_ERR_WORKSPACE,
                              "backward_w_noalloc: this call needs more scratch than the 8 MiB static array "
                              "(out_dim * K * (8 + ceil(batch/(32*vec)) * elem) too large); use clb_difflogic_backward_w");
    void* base = nullptr;
    int st = scratch_address(&base);
    if (st) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int32_t* slots = reinterpret_cast<int32_t*>(base);
    void* part = reinterpret_cast<char*>(base) + slot_bytes;

    cudaError_t e = clb::launch_slots_dense(a, b, out_dim, K, in_dim, slots, nullptr, s);
    if (e != cudaSuccess) return clb::set_error(CLB_ERR_CUDA, cudaGetErrorString(e));
    clb::LayerArgs la{};
    la.dtype = dtype;
    la.x = x;
    la.ldx = batch;
    la.ncols = batch;
    la.slots = slots;
    la.n_out = out_dim;
    la.K = (int)K;
    la.group = 1;
    la.mode = CLB_W_PROBS;
    la.gates = gate_seq;
    la.in_features = in_dim;
    if (batch > 0) {
        e = clb::launch_logic_backward(la, grad_y, batch, nullptr, nullptr, 0, part, chunks, s);
        if (e != cudaSuccess) return clb::set_error(CLB_ERR_CUDA, cudaGetErrorString(e));
    }
    e = clb::launch_grad_finalize(la, part, chunks, grad_w, dtype, s);
    if (e != cudaSuccess) return clb::set_error(CLB_ERR_CUDA, cudaGetErrorString(e));
    clb::count_launches(batch > 0 ? 3 : 2);
    return CLB_OK;
}
