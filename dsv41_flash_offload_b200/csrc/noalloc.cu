// The layer forward for callers that cannot allocate device memory.
//
// Some callers of a MoE layer cannot call cudaMalloc (or any allocator) at the moment they run the
// layer: code that runs while a CUDA graph is being captured by someone else, plugins that are
// handed a stream but no allocator by their host engine, and processes whose memory pool is fully
// reserved up front. dsv41_moe_forward needs a caller-provided workspace, which such callers do
// not have. dsv41_moe_forward_noalloc runs the same forward with its scratch in a fixed device array
// that is part of this library instead.
//
// The array (kNoAllocScratchBytes, 32 MiB) is a file-scope __device__ variable: every GPU on which
// the library is used holds it until the process exits. In host code its name is only a host-side
// stand-in, so its device address is looked up with cudaGetSymbolAddress, with the device current.
// The first call on a device does that lookup, so that first call should happen before any stream
// capture. Later calls made outside a stream capture look the address up again (it can change when
// the context is torn down and re-created, e.g. after cudaDeviceReset); calls under capture reuse the
// last address.
// All calls on a device share the array and it keeps the contents of the last call: the status word
// at its start is cleared at the beginning of every call (the split-K counters are cleared by the
// forward itself), and calls that overlap on the GPU -- on different streams, or from different
// threads -- race on it. dsv41_moe_noalloc_read_status reads (and clears) the status word.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/dsv41_b200.h"
#include "internal.h"

namespace dsv41 {

constexpr size_t kNoAllocScratchBytes = (size_t)32 << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kNoAllocMaxDevices = 64;
static void* g_noalloc_ptr[kNoAllocMaxDevices] = {nullptr};
static std::mutex g_noalloc_mutex;

// device address of the scratch array on the current device: looked up on the first call on a device
// and on every call made outside a stream capture (`stream` is not capturing)
static int noalloc_scratch(cudaStream_t stream, void** out)
{
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return set_error(DSV41_E_CUDA, "noalloc: cudaGetDevice: %s", cudaGetErrorString(err));
    if (dev < 0 || dev >= kNoAllocMaxDevices) return set_error(DSV41_E_INVALID, "noalloc: device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    bool lookup = g_noalloc_ptr[dev] == nullptr;
    if (!lookup) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        lookup = cudaStreamIsCapturing(stream, &cs) == cudaSuccess && cs == cudaStreamCaptureStatusNone;
    }
    if (lookup) {
        void* p = nullptr;
        err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (err != cudaSuccess || !p)
            return set_error(DSV41_E_CUDA, "noalloc: cudaGetSymbolAddress of the static scratch failed: %s",
                             cudaGetErrorString(err));
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return DSV41_OK;
}

}  // namespace dsv41

using namespace dsv41;

extern "C" int dsv41_moe_forward_noalloc(const dsv41_moe_layer* layer, const void* x, int32_t x_dtype, int32_t T,
                                         const int64_t* ids, const float* weights, int32_t topk,
                                         const dsv41_moe_options* opt, float* out, void* stream)
{
    // every argument is checked before anything is queued on the stream
    int rc = validate_forward(layer, x, x_dtype, T, ids, weights, topk, opt, out);
    if (rc != DSV41_OK) return rc;
    size_t need = 0;
    rc = dsv41_moe_workspace_size(T, topk, layer->num_experts, layer->hidden, layer->intermediate, opt, &need);
    if (rc != DSV41_OK) return rc;
    if (need > kNoAllocScratchBytes)
        return set_error(DSV41_E_WORKSPACE,
                         "dsv41_moe_forward_noalloc: T=%d x topk=%d at E=%d H=%d I=%d needs %zu bytes of scratch, more "
                         "than the %zu-byte static scratch; use dsv41_moe_forward with a caller workspace",
                         T, topk, layer->num_experts, layer->hidden, layer->intermediate, need, kNoAllocScratchBytes);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    void* ws = nullptr;
    if ((rc = noalloc_scratch(st, &ws)) != DSV41_OK) return rc;
    cudaError_t err = cudaMemsetAsync(ws, 0, 256, st);  // status word
    if (err != cudaSuccess) return set_error(DSV41_E_CUDA, "noalloc: clearing the status word: %s", cudaGetErrorString(err));
    return dsv41_moe_forward(layer, x, x_dtype, T, ids, weights, topk, opt, out, ws, kNoAllocScratchBytes, stream);
}

extern "C" int dsv41_moe_noalloc_read_status(void* stream, int32_t* status)
{
    if (!status) return set_error(DSV41_E_INVALID, "status is NULL");
    void* ws = nullptr;
    int rc = noalloc_scratch(static_cast<cudaStream_t>(stream), &ws);
    if (rc != DSV41_OK) return rc;
    return dsv41_read_status(ws, stream, status);
}
