// sp.cu -- carry fix-up of the sequence-parallel (T-sharded) scan.
//
// Rank r scanned its slice [r*T/P, (r+1)*T/P) from a zero state and produced,
// per channel, the slice map (A_r = prod a, B_r = h at the slice end).  With
// every rank's map gathered, the true state entering slice r is
//     carry_r = B_{r-1} + A_{r-1} * (B_{r-2} + A_{r-2} * ( ... ))
// and the slice's outputs need h[t] += (prod_{s<=t} a[s]) * carry_r.  The
// product at each tile start was recorded by the local scan (tile_prod), so
// tiles are independent: one warp per tile recomputes a (the same rounded
// gate the scan used), walks its rows and rewrites the outputs.  A tile whose
// starting correction is at most 2^-24 * |carry| on every channel is skipped
// (gated decays lie in [0, 1], so the correction only shrinks from there);
// with decays in (0, 1) only the leading ~log(2^-24)/log(mean a) tokens of a
// slice are touched.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "host_common.h"
#include "need_scan.h"
#include "scan_kernel.cuh"

using namespace need;

namespace {

struct FixParams {
    int32_t form, rowdec;
    int32_t nb, nh, T, C, L, ncb, nchains, nchunks, ntiles;
    int32_t nranks, rank;
    const void* dec;  // GATED: z; AFFINE: decay (full or per row)
    int64_t dsb, dsh, dst;
    void* out;
    int64_t osb, osh, ost;
    const uint8_t* seg;
    int64_t sgb, sgt;
    const float* tile_prod;
    const float* all_summary;
    float* h_final;
    float* summary;
};

template <typename T>
__device__ __forceinline__ void ld8f(const T* p, float (&f)[8]) {
    using O = Ops<T>;
    if constexpr (O::BYTES == 4) {
        const float4 a = *reinterpret_cast<const float4*>(p);
        const float4 b = *reinterpret_cast<const float4*>(p + 4);
        f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
        f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    } else {
        const uint4 a = *reinterpret_cast<const uint4*>(p);
        const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 v = O::unpack(*reinterpret_cast<const typename O::P*>(&w[i]));
            f[2 * i] = v.x;
            f[2 * i + 1] = v.y;
        }
    }
}

template <typename T>
__device__ __forceinline__ void st8f(T* p, const float (&f)[8]) {
    using O = Ops<T>;
    if constexpr (O::BYTES == 4) {
        *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
        *reinterpret_cast<float4*>(p + 4) = make_float4(f[4], f[5], f[6], f[7]);
    } else {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const typename O::P v = O::pack(f[2 * i], f[2 * i + 1]);
            w[i] = *reinterpret_cast<const uint32_t*>(&v);
        }
        *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// TS: dtype of out (and of z for GATED); TD: dtype of an AFFINE decay.
template <typename TS, typename TD>
__global__ void __launch_bounds__(128) fixup_kernel(const FixParams p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile = blockIdx.x * 4 + warp;
    if (tile >= p.ntiles) return;
    const int chunk = tile / p.nchains;
    const int chain = tile - chunk * p.nchains;
    const int seq = chain / p.ncb;
    const int cblk = chain - seq * p.ncb;
    const int bi = seq / p.nh, hi = seq - bi * p.nh;
    const int c = cblk * CB + lane * 8;
    const bool active = c < p.C;

    float carry[8], At[8], corr[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        carry[e] = 0.0f;
        At[e] = 1.0f;
        corr[e] = 0.0f;
    }
    bool need = false;
    if (active) {
        const size_t nsc = size_t(p.nb) * p.nh * p.C;
        for (int j = 0; j < p.rank; ++j) {
            const float2* sj = reinterpret_cast<const float2*>(p.all_summary) + j * nsc + size_t(seq) * p.C + c;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float2 m = sj[e];
                carry[e] = fmaf(m.x, carry[e], m.y);
            }
        }
        const float* tp = p.tile_prod + (size_t(seq) * p.nchunks + chunk) * p.C + c;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            corr[e] = tp[e] * carry[e];
            const bool tiny = p.form == FORM_GATED ? fabsf(corr[e]) <= 5.9604645e-8f * fabsf(carry[e])
                                                   : corr[e] == 0.0f;
            need |= !tiny;
        }
    }
    // slice summary / final state: the chunk-0 warp of each chain
    if (chunk == 0 && active) {
        const float2* mine = reinterpret_cast<const float2*>(p.all_summary) +
                             size_t(p.rank) * p.nb * p.nh * p.C + size_t(seq) * p.C + c;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float2 m = mine[e];
            const float hl = fmaf(m.x, carry[e], m.y);
            if (p.h_final) p.h_final[size_t(seq) * p.C + c + e] = hl;
            if (p.summary) reinterpret_cast<float2*>(p.summary)[size_t(seq) * p.C + c + e] = make_float2(m.x, hl);
        }
    }
    if (!__any_sync(0xffffffffu, need)) return;
    if (!active) return;

    const int t0 = chunk * p.L;
    const int nrows = min(p.L, p.T - t0);
    TS* orow = reinterpret_cast<TS*>(p.out) + bi * p.osb + hi * p.osh + c;
    for (int r = 0; r < nrows; ++r) {
        const int64_t t = t0 + r;
        const bool reset = p.seg != nullptr && p.seg[bi * p.sgb + t * p.sgt] != 0;
        float a[8];
        if (p.form == FORM_GATED) {
            float z[8];
            ld8f<TS>(reinterpret_cast<const TS*>(p.dec) + bi * p.dsb + hi * p.dsh + t * p.dst + c, z);
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
                const float2 d = Ops<TS>::unpack(Ops<TS>::pack(sigm<TS>(z[e]), sigm<TS>(z[e + 1])));
                a[e] = d.x;
                a[e + 1] = d.y;
            }
        } else if (p.rowdec) {
            const float d = to_f(reinterpret_cast<const TD*>(p.dec)[bi * p.dsb + hi * p.dsh + t * p.dst]);
#pragma unroll
            for (int e = 0; e < 8; ++e) a[e] = d;
        } else {
            ld8f<TD>(reinterpret_cast<const TD*>(p.dec) + bi * p.dsb + hi * p.dsh + t * p.dst + c, a);
        }
        float h[8];
        ld8f<TS>(orow + t * p.ost, h);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            corr[e] = (reset ? 0.0f : a[e]) * corr[e];
            h[e] += corr[e];
        }
        st8f<TS>(orow + t * p.ost, h);
    }
}

}  // namespace

extern "C" int need_sp_fixup(const need_scan_args* a, const float* all_summary, int32_t nranks, int32_t rank,
                             need_stream_t stream) {
    if (a == nullptr || all_summary == nullptr) return fail(NEED_ERR_INVALID, "null argument");
    if (a->form != NEED_FORM_GATED && a->form != NEED_FORM_AFFINE)
        return fail(NEED_ERR_UNSUPPORTED, "sequence-parallel fix-up takes the GATED or AFFINE form");
    if (nranks < 1 || rank < 0 || rank >= nranks) return fail(NEED_ERR_INVALID, "rank %d of %d", rank, nranks);
    if (a->nb < 1 || a->nh < 1 || a->T < 1 || a->C < 1) return fail(NEED_ERR_INVALID, "bad sizes");
    if (a->C % 8 != 0) return fail(NEED_ERR_UNSUPPORTED, "C must be a multiple of 8");
    if (a->tile_prod == nullptr) return fail(NEED_ERR_INVALID, "tile_prod is null (request it from the local scan)");
    if (!aligned16(a->out)) return fail(NEED_ERR_UNSUPPORTED, "out is not 16-byte aligned");
    const bool gated = a->form == NEED_FORM_GATED;
    const int rd = gated ? 0 : (a->decay_per_row ? 1 : 0);
    const int ddt = gated ? a->dtype : a->decay_dtype;
    const int64_t L = need_scan_chunk_len(a->form, a->dtype, ddt, rd);
    if (L <= 0) return fail(NEED_ERR_UNSUPPORTED, "no kernel for this dtype combination");
    const need_view& dv = a->in[0];
    if (dv.ptr == nullptr) return fail(NEED_ERR_INVALID, "in[0] is null");
    if (!rd && !aligned16(dv.ptr)) return fail(NEED_ERR_UNSUPPORTED, "in[0] is not 16-byte aligned");
    if (rank == 0) return ok();  // no carry enters the first slice

    FixParams p{};
    p.form = a->form;
    p.rowdec = rd;
    p.nb = int32_t(a->nb);
    p.nh = int32_t(a->nh);
    p.T = int32_t(a->T);
    p.C = int32_t(a->C);
    p.L = int32_t(L);
    p.ncb = int32_t((a->C + CB - 1) / CB);
    p.nchains = p.nb * p.nh * p.ncb;
    p.nchunks = int32_t((a->T + L - 1) / L);
    p.ntiles = p.nchains * p.nchunks;
    p.nranks = nranks;
    p.rank = rank;
    p.dec = dv.ptr;
    p.dsb = dv.stride_b;
    p.dsh = dv.stride_h;
    p.dst = dv.stride_t;
    p.out = a->out;
    p.osb = a->out_stride_b;
    p.osh = a->out_stride_h;
    p.ost = a->out_stride_t;
    p.seg = a->seg_start;
    p.sgb = a->seg_stride_b;
    p.sgt = a->seg_stride_t;
    p.tile_prod = a->tile_prod;
    p.all_summary = all_summary;
    p.h_final = a->h_final;
    p.summary = a->summary;
    const unsigned blocks = static_cast<unsigned>((p.ntiles + 3) / 4);
    const int dt = a->dtype;
    if (dt == NEED_BF16 && ddt == NEED_BF16) fixup_kernel<__nv_bfloat16, __nv_bfloat16><<<blocks, 128, 0, stream>>>(p);
    else if (dt == NEED_BF16 && ddt == NEED_F32) fixup_kernel<__nv_bfloat16, float><<<blocks, 128, 0, stream>>>(p);
    else if (dt == NEED_F16 && ddt == NEED_F16) fixup_kernel<__half, __half><<<blocks, 128, 0, stream>>>(p);
    else if (dt == NEED_F16 && ddt == NEED_F32) fixup_kernel<__half, float><<<blocks, 128, 0, stream>>>(p);
    else if (dt == NEED_F32 && ddt == NEED_F32) fixup_kernel<float, float><<<blocks, 128, 0, stream>>>(p);
    else return fail(NEED_ERR_UNSUPPORTED, "dtype %d / decay dtype %d", dt, ddt);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ok() : cuda_fail(e, "fixup_kernel launch");
}
