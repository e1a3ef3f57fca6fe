// epilogue.cu -- RMSNorm over the channels of each token, the SSD block's
// out_norm after its scan (need_core.py:1643), with the arithmetic of the
// reference's GPU rms_norm (need_kernels.py:99-107): per row, x widened to
// fp32, ss = sum(x^2) / C, inv = rsqrt(ss + eps), out = (x * inv) * w as two
// fp32 products, rounded once to the row's dtype.
//
// One warp per row.  The row is read in 16-byte pieces (lane l takes pieces
// l, l + 32, ...) whose squares it sums in that fixed order; a butterfly adds
// the lanes, so the result is the same on every call.  Rows of up to 256
// pieces (2048 16-bit channels) stay in registers between the sum and the
// scaling; longer rows are read a second time (from L1).  Every piece is read
// and written by the same lane, so `out` may be `x`.  Run right after the
// scan, the rows come from L2.
#include "host_common.h"
#include "need_scan.h"
#include "scan_kernel.cuh"

using namespace need;

namespace {

struct NormParams {
    const void* x;
    void* out;
    const void* w;
    int64_t xsb, xst, osb, ost;  // element strides
    int64_t T, rows;
    int32_t C, w32;
    float eps;
};

constexpr int kRowsPerBlock = 8;  // warps per block

// VPL > 0: the row is read once into registers (at most VPL 16-byte pieces per
// lane).  VPL == 0: two passes over the row, the second from L1.
template <typename TS, int VPL>
__global__ void __launch_bounds__(kRowsPerBlock * 32) rms_norm_kernel(const NormParams p) {
    using PS = typename Ops<TS>::P;
    constexpr int VEC = 16 / Ops<TS>::BYTES;
    const int lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * kRowsPerBlock + (threadIdx.x >> 5);
    if (row >= p.rows) return;
    const int64_t b = row / p.T, t = row - b * p.T;
    const TS* x = static_cast<const TS*>(p.x) + b * p.xsb + t * p.xst;
    TS* out = static_cast<TS*>(p.out) + b * p.osb + t * p.ost;
    const int nvec = p.C / VEC;

    auto sumsq = [](const uint4& u, float acc) {
        const PS* h = reinterpret_cast<const PS*>(&u);
#pragma unroll
        for (int e = 0; e < VEC / 2; ++e) {
            const float2 y = widen(h[e]);
            acc = fmaf(y.x, y.x, acc);
            acc = fmaf(y.y, y.y, acc);
        }
        return acc;
    };
    auto scale = [&](uint4 u, int v, float inv) {
        float wv[VEC];
        if (p.w32) {
            const float4* w4 = reinterpret_cast<const float4*>(static_cast<const float*>(p.w) + v * VEC);
#pragma unroll
            for (int e = 0; e < VEC / 4; ++e) {
                const float4 w = __ldg(w4 + e);
                wv[4 * e] = w.x, wv[4 * e + 1] = w.y, wv[4 * e + 2] = w.z, wv[4 * e + 3] = w.w;
            }
        } else {
            const uint4 wu = __ldg(reinterpret_cast<const uint4*>(static_cast<const TS*>(p.w) + v * VEC));
            const PS* wh = reinterpret_cast<const PS*>(&wu);
#pragma unroll
            for (int e = 0; e < VEC / 2; ++e) {
                const float2 w = widen(wh[e]);
                wv[2 * e] = w.x, wv[2 * e + 1] = w.y;
            }
        }
        PS* h = reinterpret_cast<PS*>(&u);
#pragma unroll
        for (int e = 0; e < VEC / 2; ++e) {
            const float2 y = widen(h[e]);
            h[e] = Ops<TS>::pack(__fmul_rn(__fmul_rn(y.x, inv), wv[2 * e]),
                                 __fmul_rn(__fmul_rn(y.y, inv), wv[2 * e + 1]));
        }
        *reinterpret_cast<uint4*>(out + v * VEC) = u;
    };

    float acc = 0.0f;
    if constexpr (VPL > 0) {
        uint4 u[VPL];
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            const int v = lane + 32 * k;
            if (v < nvec) u[k] = *reinterpret_cast<const uint4*>(x + v * VEC);
        }
#pragma unroll
        for (int k = 0; k < VPL; ++k)
            if (lane + 32 * k < nvec) acc = sumsq(u[k], acc);
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
        const float inv = rsqrtf(__fadd_rn(__fdiv_rn(acc, static_cast<float>(p.C)), p.eps));
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            const int v = lane + 32 * k;
            if (v < nvec) scale(u[k], v, inv);
        }
    } else {
#pragma unroll 4
        for (int v = lane; v < nvec; v += 32) acc = sumsq(*reinterpret_cast<const uint4*>(x + v * VEC), acc);
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
        const float inv = rsqrtf(__fadd_rn(__fdiv_rn(acc, static_cast<float>(p.C)), p.eps));
#pragma unroll 4
        for (int v = lane; v < nvec; v += 32) scale(*reinterpret_cast<const uint4*>(x + v * VEC), v, inv);
    }
}

template <typename TS>
void launch_norm(const NormParams& p, dim3 grid, dim3 block, cudaStream_t s) {
    const int nvec = p.C / (16 / int(sizeof(TS)));
    if (nvec <= 32) rms_norm_kernel<TS, 1><<<grid, block, 0, s>>>(p);
    else if (nvec <= 64) rms_norm_kernel<TS, 2><<<grid, block, 0, s>>>(p);
    else if (nvec <= 128) rms_norm_kernel<TS, 4><<<grid, block, 0, s>>>(p);
    else if (nvec <= 256) rms_norm_kernel<TS, 8><<<grid, block, 0, s>>>(p);
    else rms_norm_kernel<TS, 0><<<grid, block, 0, s>>>(p);
}

}  // namespace

namespace need {

int rms_norm_rows(int32_t dtype, const void* x, int64_t xsb, int64_t xst, void* out, int64_t osb, int64_t ost,
                  int64_t nb, int64_t T, int64_t C, const void* weight, int32_t weight_dtype, double eps,
                  cudaStream_t stream) {
    if (!dtype_ok(dtype)) return fail(NEED_ERR_UNSUPPORTED, "rms norm: dtype %d", dtype);
    if (x == nullptr || out == nullptr || weight == nullptr)
        return fail(NEED_ERR_INVALID, "rms norm: x, out and weight must be non-null");
    if (nb < 1 || T < 1 || C < 1) return fail(NEED_ERR_INVALID, "rms norm: sizes must be >= 1");
    if (weight_dtype != NEED_F32 && weight_dtype != dtype)
        return fail(NEED_ERR_UNSUPPORTED, "rms norm: weight dtype %d must be fp32 or %d", weight_dtype, dtype);
    if (!(eps >= 0.0)) return fail(NEED_ERR_INVALID, "rms norm: eps must be >= 0");
    const int64_t vec = 16 / dtype_bytes(dtype);
    if (C % vec != 0 || C > INT32_MAX / 2)
        return fail(NEED_ERR_UNSUPPORTED, "rms norm: C=%lld must be a multiple of %lld", (long long)C,
                    (long long)vec);
    if (!aligned16(x) || !aligned16(out) || !aligned16(weight))
        return fail(NEED_ERR_UNSUPPORTED, "rms norm: x, out and weight must be 16-byte aligned");
    if ((T > 1 && (xst % vec != 0 || ost % vec != 0)) || (nb > 1 && (xsb % vec != 0 || osb % vec != 0)))
        return fail(NEED_ERR_UNSUPPORTED, "rms norm: row strides must be multiples of %lld elements", (long long)vec);
    NormParams p{x, out, weight, xsb, xst, osb, ost, T, nb * T, static_cast<int32_t>(C),
                 weight_dtype == NEED_F32 ? 1 : 0, static_cast<float>(eps)};
    const int64_t blocks = (p.rows + kRowsPerBlock - 1) / kRowsPerBlock;
    if (blocks > INT32_MAX) return fail(NEED_ERR_UNSUPPORTED, "rms norm: too many rows");
    const dim3 grid(static_cast<unsigned>(blocks)), block(kRowsPerBlock * 32);
    if (dtype == NEED_BF16) launch_norm<__nv_bfloat16>(p, grid, block, stream);
    else if (dtype == NEED_F16) launch_norm<__half>(p, grid, block, stream);
    else launch_norm<float>(p, grid, block, stream);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "rms_norm_kernel launch");
    return NEED_OK;
}

}  // namespace need

extern "C" int need_rms_norm(const need_norm_args* a, need_stream_t stream) {
    if (a == nullptr) return fail(NEED_ERR_INVALID, "args is null");
    if (int rc = rms_norm_rows(a->dtype, a->x, a->x_stride_b, a->x_stride_t, a->out, a->out_stride_b,
                               a->out_stride_t, a->nb, a->T, a->C, a->weight, a->weight_dtype, a->eps, stream))
        return rc;
    return ok();
}
