// decode.cu -- ragged decode / speculative-verify state update and commit.
//
// need_ragged_verify runs k_i one-token recurrent steps for each of nseq
// sequences from its pooled state, in the model dtype's arithmetic of the
// reference's streaming steps (need_core.py:6420-6428 for the SSD / gated
// block, :1590-1592 and :6440-6444 for SelectiveRetention: every op rounded to
// the state dtype), and records the output and the state after every drafted
// token.  need_commit_states then keeps, per sequence, the state after its
// accepted prefix (the reference keeps the accepted tokens, generate.py:1078-1083,
// and recomputes its whole context on the next verify, generate.py:909-913).
//
// The SSD form optionally runs the block's causal depthwise conv per drafted
// token (need_core.py:6395-6414, _stream_depthwise_conv1d_step and SiLU) from
// each sequence's conv history, and records the history after every token so
// that a commit can keep it at the accepted prefix together with the state.
//
// One thread owns 8 channels of one sequence; a sequence's drafted tokens are
// processed four at a time with all their loads issued before the dependent
// arithmetic.  Both kernels are latency-bound (a decode step moves ~12 MB at
// 256 sequences x 1024 channels); callers capture them in a CUDA graph.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "host_common.h"
#include "need_scan.h"
#include "scan_kernel.cuh"

using namespace need;

namespace {

struct VerifyParams {
    int64_t nseq, C;
    void* states;
    const int32_t* slot;
    const int32_t* cu_k;
    const void* in[5];
    const float* dskip;
    float dt_min, dt_scale;
    void* y;
    void* states_k;
    int64_t H, head_dim;  // RETENTION: in[0] is the decay per (token, head) [sum k, H]
    // SSD with the conv step: weight [C, K], bias [C] or null, history [nslots, C, K-1]
    // (read) and after every drafted token [total_k, C, K-1] (written)
    const void* conv_w;
    const void* conv_b;
    const void* conv_hist;
    void* conv_hist_k;
};

template <typename T>
struct Vec8 {
    using P = typename Ops<T>::P;
    // 8 consecutive elements as 4 pairs
    static __device__ __forceinline__ void ld(const T* p, P (&v)[4]) {
        if constexpr (Ops<T>::BYTES == 4) {
            const float4 a = *reinterpret_cast<const float4*>(p);
            const float4 b = *reinterpret_cast<const float4*>(p + 4);
            v[0] = make_float2(a.x, a.y);
            v[1] = make_float2(a.z, a.w);
            v[2] = make_float2(b.x, b.y);
            v[3] = make_float2(b.z, b.w);
        } else {
            const uint4 a = *reinterpret_cast<const uint4*>(p);
            const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] = *reinterpret_cast<const P*>(&w[i]);
        }
    }
    static __device__ __forceinline__ void st(T* p, const P (&v)[4]) {
        if constexpr (Ops<T>::BYTES == 4) {
            *reinterpret_cast<float4*>(p) = make_float4(v[0].x, v[0].y, v[1].x, v[1].y);
            *reinterpret_cast<float4*>(p + 4) = make_float4(v[2].x, v[2].y, v[3].x, v[3].y);
        } else {
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) w[i] = *reinterpret_cast<const uint32_t*>(&v[i]);
            *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
};

// x / (1 + exp(-x)) in fp32, rounded to T: SiLU at the reference's rounding
// points (the 16-bit paths use the hardware exp2 approximation, a few ulp)
template <typename T>
__device__ __forceinline__ float silu_rounded(float x) {
    float d;
    if constexpr (Ops<T>::BYTES == 4) d = __fadd_rn(1.0f, expf(-x));
    else d = __fadd_rn(1.0f, exp_approx(-x));
    const float r = __fdiv_rn(x, d);
    if constexpr (Ops<T>::BYTES == 4) return r;
    else return to_f(Ops<T>::pack(r, r).x);
}

template <typename T>
__device__ __forceinline__ float rnd_to(float x) {
    if constexpr (Ops<T>::BYTES == 4) return x;
    else return to_f(Ops<T>::pack(x, x).x);
}

// KC: conv taps of the SSD form's conv step (0: in[2] is already u_act)
template <typename T, int FORM, int KC = 0>
__global__ void __launch_bounds__(128) verify_kernel(const VerifyParams p) {
    using O = Ops<T>;
    using P = typename O::P;
    constexpr int KH = KC > 1 ? KC - 1 : 1;  // history taps kept per channel
    constexpr int TB = KC > 0 ? 2 : 4;       // drafted tokens loaded together (fewer with the conv state)
    // streamed [C] inputs: GATED z, g, x; SSD dt, bg, u, cg, og; RETENTION k, v, q (in[1..3])
    constexpr int NIN = FORM == FORM_SSD ? 5 : 3;
    constexpr int IN0 = FORM == FORM_RETENTION ? 1 : 0;
    const int64_t i = blockIdx.y;
    const int64_t c = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
    if (i >= p.nseq || c >= p.C) return;
    const int64_t row = p.slot ? p.slot[i] : i;
    const int64_t kb = p.cu_k[i], ke = p.cu_k[i + 1];
    P st[4];
    Vec8<T>::ld(reinterpret_cast<const T*>(p.states) + row * p.C + c, st);
    P dsk[4];
    if constexpr (FORM == FORM_SSD) {
#pragma unroll
        for (int q = 0; q < 4; ++q) dsk[q] = O::pack(p.dskip[c + 2 * q], p.dskip[c + 2 * q + 1]);
    }
    const int64_t head = FORM == FORM_RETENTION ? c / p.head_dim : 0;  // a thread's 8 channels share a head
    // conv step state: this thread's 8 channels' weights, bias and history
    float cw[8][KC > 0 ? KC : 1], cb[8], hist[8][KH];
    if constexpr (KC > 0) {
        const T* w = static_cast<const T*>(p.conv_w) + c * KC;
        const T* hs = static_cast<const T*>(p.conv_hist) + (row * p.C + c) * (KC - 1);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            cb[e] = p.conv_b != nullptr ? to_f(static_cast<const T*>(p.conv_b)[c + e]) : 0.0f;
#pragma unroll
            for (int j = 0; j < KC; ++j) cw[e][j] = to_f(w[e * KC + j]);
#pragma unroll
            for (int j = 0; j < KC - 1; ++j) hist[e][j] = to_f(hs[e * (KC - 1) + j]);
        }
    }
    for (int64_t j0 = kb; j0 < ke; j0 += TB) {
        P x[TB][NIN][4];
        T dh[TB];
#pragma unroll
        for (int u = 0; u < TB; ++u)
            if (j0 + u < ke) {
#pragma unroll
                for (int k = 0; k < NIN; ++k)
                    Vec8<T>::ld(reinterpret_cast<const T*>(p.in[IN0 + k]) + (j0 + u) * p.C + c, x[u][k]);
                if constexpr (FORM == FORM_RETENTION) dh[u] = reinterpret_cast<const T*>(p.in[0])[(j0 + u) * p.H + head];
            }
#pragma unroll
        for (int u = 0; u < TB; ++u) {
            if (j0 + u >= ke) break;
            P yo[4];
            if constexpr (FORM == FORM_RETENTION) {
                // need_core.py:1590-1592: state = decay * state + k * v; y = q * state,
                // each op in the state dtype
                const float df = to_f(dh[u]);
                const P dec = O::pack(df, df);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    st[q] = O::add(O::mul(dec, st[q]), O::mul(x[u][0][q], x[u][1][q]));
                    yo[q] = O::mul(x[u][2][q], st[q]);
                }
            } else {
                if constexpr (KC > 0) {
                    // need_core.py:6395-6409, :6413-6414: u_act = silu(conv step), in[2] raw u
                    T* hk = static_cast<T*>(p.conv_hist_k) + ((j0 + u) * p.C + c) * (KC - 1);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float2 ur = O::unpack(x[u][2][q]);
                        float ua[2];
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const int e = 2 * q + h;
                            const float un = h ? ur.y : ur.x;
                            float acc = 0.0f;
#pragma unroll
                            for (int j = 0; j < KC; ++j)
                                acc = __fadd_rn(acc, rnd_to<T>(__fmul_rn(j < KC - 1 ? hist[e][j] : un, cw[e][j])));
                            float uc = rnd_to<T>(acc);
                            if (p.conv_b != nullptr) uc = rnd_to<T>(__fadd_rn(uc, cb[e]));
#pragma unroll
                            for (int j = 0; j + 1 < KC - 1; ++j) hist[e][j] = hist[e][j + 1];
                            hist[e][KC - 2] = un;
                            ua[h] = silu_rounded<T>(uc);
                        }
                        x[u][2][q] = O::pack(ua[0], ua[1]);
                    }
#pragma unroll
                    for (int e = 0; e < 8; ++e)
#pragma unroll
                        for (int j = 0; j < KC - 1; ++j) hk[e * (KC - 1) + j] = O::pack(hist[e][j], 0.0f).x;
                }
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float2 f0 = O::unpack(x[u][0][q]);
                    const float2 f1 = O::unpack(x[u][1][q]);
                    P dec;
                    if constexpr (FORM == FORM_GATED) {
                        dec = O::pack(sigm<T>(f0.x), sigm<T>(f0.y));
                    } else {
                        const float dx = __fadd_rn(__fmul_rn(sigm<T>(f0.x), p.dt_scale), p.dt_min);
                        const float dy = __fadd_rn(__fmul_rn(sigm<T>(f0.y), p.dt_scale), p.dt_min);
                        dec = O::pack(expo<T>(-dx), expo<T>(-dy));
                    }
                    const P gs = O::pack(sigm<T>(f1.x), sigm<T>(f1.y));
                    // rec = decay * rec + (1 - decay) * (bg * u)
                    st[q] = O::add(O::mul(dec, st[q]), O::mul(O::sub(O::one(), dec), O::mul(gs, x[u][2][q])));
                    if constexpr (FORM == FORM_GATED) {
                        yo[q] = st[q];
                    } else {
                        const float2 f3 = O::unpack(x[u][3][q]);
                        const float2 f4 = O::unpack(x[u][4][q]);
                        const P cgs = O::pack(sigm<T>(f3.x), sigm<T>(f3.y));
                        const P ogs = O::pack(sigm<T>(f4.x), sigm<T>(f4.y));
                        yo[q] = O::mul(O::add(O::mul(cgs, st[q]), O::mul(dsk[q], x[u][2][q])), ogs);
                    }
                }
            }
            Vec8<T>::st(reinterpret_cast<T*>(p.y) + (j0 + u) * p.C + c, yo);
            Vec8<T>::st(reinterpret_cast<T*>(p.states_k) + (j0 + u) * p.C + c, st);
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(128) commit_kernel(int64_t nseq, int64_t C, T* states, const int32_t* slot,
                                                     const T* states_k, const int32_t* cu_k,
                                                     const int32_t* accept) {
    const int64_t i = blockIdx.y;
    const int64_t c = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
    if (i >= nseq || c >= C) return;
    const int64_t kb = cu_k[i], ke = cu_k[i + 1];
    int64_t L = accept[i];
    L = L < 0 ? 0 : (L > ke - kb ? ke - kb : L);
    if (L == 0) return;
    const int64_t row = slot ? slot[i] : i;
    typename Ops<T>::P v[4];
    Vec8<T>::ld(states_k + (kb + L - 1) * C + c, v);
    Vec8<T>::st(states + row * C + c, v);
}

dim3 grid_for(int64_t nseq, int64_t C) {
    const int64_t vecs = C / 8;
    return dim3(static_cast<unsigned>((vecs + 127) / 128), static_cast<unsigned>(nseq));
}

int check_rows(int dtype, int64_t nseq, int64_t C) {
    if (!dtype_ok(dtype)) return fail(NEED_ERR_UNSUPPORTED, "dtype %d", dtype);
    if (nseq < 0 || C < 1) return fail(NEED_ERR_INVALID, "nseq=%lld C=%lld", (long long)nseq, (long long)C);
    if (C % 8 != 0) return fail(NEED_ERR_UNSUPPORTED, "C=%lld must be a multiple of 8", (long long)C);
    if (nseq > 65535) return fail(NEED_ERR_UNSUPPORTED, "nseq=%lld exceeds 65535", (long long)nseq);
    return NEED_OK;
}

template <typename T, int FORM, int KC = 0>
int launch_verify(const VerifyParams& p, cudaStream_t s) {
    verify_kernel<T, FORM, KC><<<grid_for(p.nseq, p.C), 128, 0, s>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? NEED_OK : cuda_fail(e, "verify_kernel launch");
}

}  // namespace

extern "C" {

int need_ragged_verify(const need_verify_args* a, need_stream_t stream) {
    if (a == nullptr) return fail(NEED_ERR_INVALID, "args is null");
    if (a->form != NEED_FORM_GATED && a->form != NEED_FORM_SSD && a->form != NEED_FORM_RETENTION)
        return fail(NEED_ERR_INVALID, "form must be GATED, SSD or RETENTION");
    if (int rc = check_rows(a->dtype, a->nseq, a->C)) return rc;
    if (a->form == NEED_FORM_RETENTION &&
        (a->head_dim < 8 || a->head_dim % 8 != 0 || a->C % a->head_dim != 0))
        return fail(NEED_ERR_UNSUPPORTED, "head_dim=%lld must be a multiple of 8 that divides C=%lld",
                    (long long)a->head_dim, (long long)a->C);
    if (a->nseq == 0 || a->total_k == 0) return ok();
    const int nin = a->form == NEED_FORM_SSD ? 5 : a->form == NEED_FORM_RETENTION ? 4 : 3;
    if (!a->states || !a->cu_k || !a->y || !a->states_k) return fail(NEED_ERR_INVALID, "null pointer");
    for (int k = 0; k < nin; ++k)
        if (!a->in[k] || (!aligned16(a->in[k]) && !(a->form == NEED_FORM_RETENTION && k == 0)))
            return fail(NEED_ERR_INVALID, "in[%d] null or not 16-byte aligned", k);
    if (!aligned16(a->states) || !aligned16(a->y) || !aligned16(a->states_k))
        return fail(NEED_ERR_UNSUPPORTED, "states / y / states_k must be 16-byte aligned");
    if (a->form == NEED_FORM_SSD && !a->d_skip) return fail(NEED_ERR_INVALID, "d_skip is null");
    const int kc = a->conv_k;
    if (kc != 0) {
        if (a->form != NEED_FORM_SSD) return fail(NEED_ERR_INVALID, "conv_k is for the SSD form only");
        if (kc < 2 || kc > 4) return fail(NEED_ERR_UNSUPPORTED, "conv_k=%d must be 0 or 2..4", kc);
        if (!a->conv_weight || !a->conv_hist || !a->conv_hist_k)
            return fail(NEED_ERR_INVALID, "conv_weight, conv_hist and conv_hist_k are required with conv_k");
    }
    VerifyParams p{};
    p.nseq = a->nseq;
    p.C = a->C;
    p.states = a->states;
    p.slot = a->slot;
    p.cu_k = a->cu_k;
    for (int k = 0; k < 5; ++k) p.in[k] = a->in[k];
    p.dskip = a->d_skip;
    p.dt_min = static_cast<float>(a->dt_min);
    p.dt_scale = static_cast<float>(a->dt_max - a->dt_min);
    p.y = a->y;
    p.states_k = a->states_k;
    p.head_dim = a->form == NEED_FORM_RETENTION ? a->head_dim : 8;
    p.H = a->C / p.head_dim;
    p.conv_w = a->conv_weight;
    p.conv_b = a->conv_bias;
    p.conv_hist = a->conv_hist;
    p.conv_hist_k = a->conv_hist_k;
    const cudaStream_t s = stream;
    int rc;
    auto by_form = [&](auto tag) {
        using T = decltype(tag);
        if (a->form == NEED_FORM_SSD)
            return kc == 2 ? launch_verify<T, FORM_SSD, 2>(p, s)
                   : kc == 3 ? launch_verify<T, FORM_SSD, 3>(p, s)
                   : kc == 4 ? launch_verify<T, FORM_SSD, 4>(p, s)
                             : launch_verify<T, FORM_SSD>(p, s);
        return a->form == NEED_FORM_GATED ? launch_verify<T, FORM_GATED>(p, s)
                                          : launch_verify<T, FORM_RETENTION>(p, s);
    };
    if (a->dtype == NEED_BF16) rc = by_form(__nv_bfloat16{});
    else if (a->dtype == NEED_F16) rc = by_form(__half{});
    else rc = by_form(float{});
    return rc ? rc : ok();
}

int need_commit_states(int32_t dtype, int64_t nseq, int64_t C, void* states, const int32_t* slot,
                       const void* states_k, const int32_t* cu_k, const int32_t* accept_len, need_stream_t stream) {
    if (int rc = check_rows(dtype, nseq, C)) return rc;
    if (nseq == 0) return ok();
    if (!states || !states_k || !cu_k || !accept_len) return fail(NEED_ERR_INVALID, "null pointer");
    if (!aligned16(states) || !aligned16(states_k)) return fail(NEED_ERR_UNSUPPORTED, "states must be 16-byte aligned");
    const dim3 g = grid_for(nseq, C);
    if (dtype == NEED_BF16)
        commit_kernel<__nv_bfloat16><<<g, 128, 0, stream>>>(nseq, C, static_cast<__nv_bfloat16*>(states), slot,
                                                             static_cast<const __nv_bfloat16*>(states_k), cu_k, accept_len);
    else if (dtype == NEED_F16)
        commit_kernel<__half><<<g, 128, 0, stream>>>(nseq, C, static_cast<__half*>(states), slot,
                                                      static_cast<const __half*>(states_k), cu_k, accept_len);
    else
        commit_kernel<float><<<g, 128, 0, stream>>>(nseq, C, static_cast<float*>(states), slot,
                                                     static_cast<const float*>(states_k), cu_k, accept_len);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ok() : cuda_fail(e, "commit_kernel launch");
}

}  // extern "C"
