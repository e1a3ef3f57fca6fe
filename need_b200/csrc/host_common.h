// host_common.h -- shared host-side helpers of the C ABI: error reporting,
// per-device one-time kernel attributes, the driver entry points the TMA
// descriptors need.
#pragma once

#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

#include <atomic>
#include <mutex>
#include <string>

#include "need_scan.h"

namespace need {

// Message of the calling thread's last failure.
inline std::string& last_error_slot() {
    static thread_local std::string msg;
    return msg;
}

inline int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    last_error_slot() = buf;
    return code;
}

inline int ok() {
    last_error_slot().clear();
    return NEED_OK;
}

inline int cuda_fail(cudaError_t e, const char* what) {
    return fail(NEED_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Per-device caches (shared-memory opt-in masks, grid sizes) cover ordinals below this.
constexpr int kMaxDevices = 64;

// Raises a kernel's dynamic shared-memory limit once per device.
template <typename Kern>
inline cudaError_t ensure_smem(Kern kern, int bytes, std::atomic<uint64_t>& done_mask) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = dev < 64 ? (uint64_t(1) << dev) : 0;
    if (bit && (done_mask.load(std::memory_order_acquire) & bit)) return cudaSuccess;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess && bit) done_mask.fetch_or(bit, std::memory_order_acq_rel);
    return e;
}

// The driver's tensor-map encoder (null when the driver lacks it).
inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// Binds the current device's primary context to the calling thread when no
// context is current there.  The tensor-map encoder is a driver call and needs
// one; a thread that has made no runtime call yet (e.g. the autograd engine's
// worker running a backward) has none until the runtime binds it lazily.
inline int ensure_context() {
    static PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 4000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
    });
    CUcontext ctx = nullptr;
    if (get_current != nullptr && get_current(&ctx) == CUDA_SUCCESS && ctx != nullptr) return NEED_OK;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaSetDevice(dev);  // initialises and binds the primary context
    return e == cudaSuccess ? NEED_OK : cuda_fail(e, "binding the device context");
}

// RMSNorm over the C channels of nb x T rows (epilogue.cu); launches only.
int rms_norm_rows(int32_t dtype, const void* x, int64_t xsb, int64_t xst, void* out, int64_t osb, int64_t ost,
                  int64_t nb, int64_t T, int64_t C, const void* weight, int32_t weight_dtype, double eps,
                  cudaStream_t stream);

inline int dtype_bytes(int dt) { return dt == NEED_F32 ? 4 : 2; }
inline bool dtype_ok(int dt) { return dt == NEED_F32 || dt == NEED_BF16 || dt == NEED_F16; }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace need
