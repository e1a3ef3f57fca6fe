// prologue.cu -- the SSD block's input prologue, fused: u = SiLU(causal
// depthwise conv_K(u_raw)) (need_core.py:1620-1622: nn.Conv1d(d, d, K,
// padding=K-1, groups=d), trimmed to the first T outputs, then F.silu).
//
// out[b, t, c] = silu(round(bias[c] + sum_j w[c, j] * u[b, t-K+1+j, c]))
// with u[t'] = 0 for t' < 0 and, when a reset mask is given, for t' before the
// segment start of t (the scan's packed-segment resets, which the conv must
// honour too).  The conv is accumulated in fp32 and rounded to the input dtype
// before SiLU, SiLU is computed in fp32 (hardware exp2 / reciprocal
// approximations, a few fp32 ulp) and rounded again: the reference's two
// rounding points.
//
// HBM-bound (2 + 2 bytes per element for 16-bit data): one thread walks 32
// tokens of 8 consecutive channels (16-byte loads and stores, 8 rows loaded
// before they are used), carrying the last K-1 raw inputs in registers;
// consecutive threads take consecutive channel groups, so a warp's loads of
// one row are contiguous.  128-thread blocks keep 3 blocks per SM resident at
// this kernel's register count; at NEED's model shape the grid then fits in
// one wave (32 tokens per thread measured 16.4 us against 18.5 us for 16).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "host_common.h"
#include "need_scan.h"
#include "scan_kernel.cuh"

using namespace need;

namespace {

#ifndef NEED_CONV_TT
#define NEED_CONV_TT 32
#endif
#ifndef NEED_CONV_GROUP
#define NEED_CONV_GROUP 8
#endif
constexpr int kConvTT = NEED_CONV_TT;       // tokens per thread
constexpr int kConvGroup = NEED_CONV_GROUP;  // rows loaded together
constexpr int kMaxTaps = 4;

struct ConvParams {
    const void* u;
    int64_t usb, ust;
    void* out;
    int64_t osb, ost;
    const void* w;      // [C, K] (element strides wsc, wsk)
    int64_t wsc, wsk;
    const void* bias;   // [C] or null
    const uint8_t* seg;
    int64_t sgb, sgt;
    int32_t nb, T, C;
};

template <typename T>
__device__ __forceinline__ float ldf(const T* p, int64_t i) { return to_f(p[i]); }

template <typename T>
__device__ __forceinline__ float round_to(float x) {
    if constexpr (Ops<T>::BYTES == 4) return x;
    else return to_f(Ops<T>::pack(x, x).x);
}

// x * sigmoid(x) with the scan's 16-bit sigmoid (ex2.approx + rcp.approx, a
// few fp32 ulp): the result is rounded to bf16 / f16 next
__device__ __forceinline__ float silu_f32(float x) { return x * sigmoid_approx(x); }

template <typename T, int K>
__global__ void __launch_bounds__(128) conv_silu_kernel(const ConvParams p) {
    constexpr int H = K > 1 ? K - 1 : 1;  // window rows kept (at least one, unused when K == 1)
    const int groups = p.C / 8;
    const int64_t nt = (p.T + kConvTT - 1) / kConvTT;
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= int64_t(p.nb) * nt * groups) return;
    const int cg = static_cast<int>(i % groups);
    const int64_t rest = i / groups;
    const int tc = static_cast<int>(rest % nt);
    const int b = static_cast<int>(rest / nt);
    const int c0 = cg * 8, t0 = tc * kConvTT;
    const T* u = static_cast<const T*>(p.u) + b * p.usb + c0;
    T* out = static_cast<T*>(p.out) + b * p.osb + c0;
    const T* w = static_cast<const T*>(p.w);

    float wt[8][K], bs[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        bs[e] = p.bias != nullptr ? ldf(static_cast<const T*>(p.bias), c0 + e) : 0.0f;
#pragma unroll
        for (int j = 0; j < K; ++j) wt[e][j] = ldf(w, (c0 + e) * p.wsc + j * p.wsk);
    }
    // window[j][e]: raw input j+1 rows before the current one (0 outside the segment)
    float win[H][8];
#pragma unroll
    for (int j = 0; j < H; ++j)
#pragma unroll
        for (int e = 0; e < 8; ++e) win[j][e] = 0.0f;
    // the K-1 rows before this thread's first token, oldest first; a reset at
    // a later row of them drops the older ones
#pragma unroll
    for (int d = K - 1; d >= 1; --d) {
        const int t = t0 - d;
        if (t < 0) continue;
        if (p.seg != nullptr && p.seg[b * p.sgb + int64_t(t) * p.sgt] != 0) {
#pragma unroll
            for (int j = 0; j < H; ++j)
#pragma unroll
                for (int e = 0; e < 8; ++e) win[j][e] = 0.0f;
        }
        typename Ops<T>::P v[4];
        Row8<T, false>::lds(u + int64_t(t) * p.ust, 0, v);
#pragma unroll
        for (int j = H - 1; j >= 1; --j)
#pragma unroll
            for (int e = 0; e < 8; ++e) win[j][e] = win[j - 1][e];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float2 f = Ops<T>::unpack(v[q]);
            win[0][2 * q] = f.x;
            win[0][2 * q + 1] = f.y;
        }
    }
    const int tend = min(t0 + kConvTT, p.T);
    // rows are loaded kConvGroup at a time, so that many loads are in flight
    // before the (sequential) window arithmetic consumes them
    for (int tg = t0; tg < tend; tg += kConvGroup) {
        typename Ops<T>::P v[kConvGroup][4];
        uint8_t rs[kConvGroup];
#pragma unroll
        for (int g = 0; g < kConvGroup; ++g) {
            const int t = tg + g;
            rs[g] = 0;
            if (t < tend) {
                Row8<T, false>::lds(u + int64_t(t) * p.ust, 0, v[g]);
                if (p.seg != nullptr) rs[g] = p.seg[b * p.sgb + int64_t(t) * p.sgt];
            }
        }
#pragma unroll
        for (int g = 0; g < kConvGroup; ++g) {
            const int t = tg + g;
            if (t >= tend) break;
            if (rs[g] != 0) {  // a segment starts here: nothing before it feeds the conv
#pragma unroll
                for (int j = 0; j < H; ++j)
#pragma unroll
                    for (int e = 0; e < 8; ++e) win[j][e] = 0.0f;
            }
            float x[8];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float2 f = Ops<T>::unpack(v[g][q]);
                x[2 * q] = f.x;
                x[2 * q + 1] = f.y;
            }
            typename Ops<T>::P o[4];
            float y[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                // taps oldest first: w[K-1] multiplies the current token
                float acc = bs[e];
#pragma unroll
                for (int j = 0; j < K; ++j) {
                    const int back = K - 1 - j;  // rows before the current one
                    acc = fmaf(wt[e][j], back == 0 ? x[e] : win[back - 1][e], acc);
                }
                y[e] = round_to<T>(silu_f32(round_to<T>(acc)));
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) o[q] = Ops<T>::pack(y[2 * q], y[2 * q + 1]);
            Row8<T, false>::sts(out + int64_t(t) * p.ost, 0, o);
#pragma unroll
            for (int j = H - 1; j >= 1; --j)
#pragma unroll
                for (int e = 0; e < 8; ++e) win[j][e] = win[j - 1][e];
#pragma unroll
            for (int e = 0; e < 8; ++e) win[0][e] = x[e];
        }
    }
}

}  // namespace

extern "C" int need_ssd_conv_silu(const need_conv_args* a, need_stream_t stream) {
    if (a == nullptr || a->u == nullptr || a->out == nullptr || a->weight == nullptr)
        return fail(NEED_ERR_INVALID, "null argument");
    if (a->nb < 1 || a->T < 1 || a->C < 1) return fail(NEED_ERR_INVALID, "sizes must be >= 1");
    if (a->K < 1 || a->K > kMaxTaps) return fail(NEED_ERR_UNSUPPORTED, "K=%d taps (1..%d supported)", a->K, kMaxTaps);
    if (a->dtype != NEED_BF16 && a->dtype != NEED_F16)
        return fail(NEED_ERR_UNSUPPORTED, "the conv prologue takes bf16 or f16 data");
    if (a->C % 8 != 0) return fail(NEED_ERR_UNSUPPORTED, "C=%lld must be a multiple of 8", (long long)a->C);
    if (!aligned16(a->u) || !aligned16(a->out) || (a->u_stride_t * 2) % 16 != 0 || (a->out_stride_t * 2) % 16 != 0 ||
        (a->u_stride_b * 2) % 16 != 0 || (a->out_stride_b * 2) % 16 != 0)
        return fail(NEED_ERR_UNSUPPORTED, "u and out need 16-byte aligned rows");
    if (a->nb * a->T > INT32_MAX || a->C > INT32_MAX) return fail(NEED_ERR_UNSUPPORTED, "sizes too large");
    ConvParams p{a->u, a->u_stride_b, a->u_stride_t, a->out, a->out_stride_b, a->out_stride_t,
                 a->weight, a->w_stride_c, a->w_stride_k, a->bias, a->seg_start, a->seg_stride_b,
                 a->seg_stride_t, int32_t(a->nb), int32_t(a->T), int32_t(a->C)};
    const int64_t threads = a->nb * ((a->T + kConvTT - 1) / kConvTT) * (a->C / 8);
    const unsigned blocks = static_cast<unsigned>((threads + 127) / 128);
    auto launch = [&](auto tag) {
        using T = decltype(tag);
        switch (a->K) {
            case 1: conv_silu_kernel<T, 1><<<blocks, 128, 0, stream>>>(p); break;
            case 2: conv_silu_kernel<T, 2><<<blocks, 128, 0, stream>>>(p); break;
            case 3: conv_silu_kernel<T, 3><<<blocks, 128, 0, stream>>>(p); break;
            default: conv_silu_kernel<T, 4><<<blocks, 128, 0, stream>>>(p); break;
        }
    };
    if (a->dtype == NEED_BF16) launch(__nv_bfloat16{});
    else launch(__half{});
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ok() : cuda_fail(e, "conv_silu_kernel launch");
}
