// noalloc.cu -- need_gated_scan with its look-back scratch in a static device
// array, for callers that cannot allocate device memory where they run the
// scan (see need_gated_scan_noalloc in need_scan.h).
#include <cuda_runtime.h>

#include <mutex>

#include "host_common.h"
#include "need_scan.h"

namespace {

constexpr size_t kScratchBytes = NEED_GATED_SCAN_NOALLOC_SCRATCH_BYTES;
constexpr size_t kErrorWordOffset = 3 * sizeof(uint32_t);  // header word 3: device error bits

// One copy per device, alive until the process exits.  Host code must not use
// this name as an address: it is a host-side stand-in; the device address
// comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_scratch on the current device.  The first call on a
// device looks the address up and zero-fills the array with cudaMemsetAsync on
// `stream`, so the fill is ordered before that call's launch on any stream
// (the look-back records must start untagged).  The address is kept for the
// life of the process: after cudaDeviceReset it is stale, and the entry points
// must not be used again in that process.
int scratch_address(cudaStream_t stream, void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return need::cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) return need::fail(NEED_ERR_UNSUPPORTED, "device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_scratch_ptr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_scratch);
        if (e != cudaSuccess) return need::cuda_fail(e, "cudaGetSymbolAddress(scratch)");
        e = cudaMemsetAsync(p, 0, kScratchBytes, stream);
        if (e != cudaSuccess) return need::cuda_fail(e, "cudaMemsetAsync(scratch)");
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return NEED_OK;
}

}  // namespace

extern "C" int need_gated_scan_noalloc(const need_scan_args* args, need_stream_t stream) {
    if (args == nullptr) return need::fail(NEED_ERR_INVALID, "args is null");
    if (args->form != NEED_FORM_GATED) return need::fail(NEED_ERR_INVALID, "args->form must be NEED_FORM_GATED");
    const size_t need = need_scan_workspace_size(args->form, args->dtype, args->dtype, 0, args->nb, args->nh,
                                                 args->T, args->C);
    if (need == 0) return need::fail(NEED_ERR_UNSUPPORTED, "no kernel for dtype %d", args->dtype);
    if (need > kScratchBytes) {
        // one tile of this plan: its records are the workspace of a 1 x 1 x 1 scan past the header
        const size_t tile_bytes = need_scan_workspace_size(args->form, args->dtype, args->dtype, 0, 1, 1, 1, 1) - 128;
        return need::fail(NEED_ERR_WORKSPACE,
                          "this scan needs %zu bytes of scratch; the static array holds %zu (at most %zu tiles "
                          "of %zu channels x %lld tokens); use need_gated_scan with a workspace",
                          need, kScratchBytes, (kScratchBytes - 128) / tile_bytes, tile_bytes / 32,
                          static_cast<long long>(need_scan_chunk_len(args->form, args->dtype, args->dtype, 0)));
    }
    void* scratch = nullptr;
    if (int rc = scratch_address(static_cast<cudaStream_t>(stream), &scratch)) return rc;
    // a bounded wait that gave up in an earlier call must not shorten this call's waits
    const cudaError_t e =
        cudaMemsetAsync(static_cast<unsigned char*>(scratch) + kErrorWordOffset, 0, sizeof(uint32_t), stream);
    if (e != cudaSuccess) return need::cuda_fail(e, "cudaMemsetAsync(scratch error word)");
    need_scan_args a = *args;
    a.workspace = scratch;
    a.workspace_bytes = kScratchBytes;
    return need_gated_scan(&a, stream);
}

extern "C" int need_gated_scan_noalloc_error(uint32_t* error_out, need_stream_t stream) {
    if (error_out == nullptr) return need::fail(NEED_ERR_INVALID, "error_out is null");
    void* scratch = nullptr;
    if (int rc = scratch_address(static_cast<cudaStream_t>(stream), &scratch)) return rc;
    // the array's workspace header holds the error word where a caller's workspace does
    return need_workspace_error(scratch, error_out, stream);
}
