// sp.cu -- carry fix-up of the sequence-parallel (T-sharded) scan.
//
// Rank r scanned its slice [r*T/P, (r+1)*T/P) from a zero state and produced,
// per channel, the slice map (A_r = prod a, B_r = h at the slice end), plus for
// every tile the product of a before it (tile_prod) and the state entering it
// (tile_carry).  With every rank's map gathered, the true state entering
// slice r is
//     carry_r = B_{r-1} + A_{r-1} * (B_{r-2} + A_{r-2} * ( ... ))
// and the state entering tile k of the slice is tile_carry[k] +
// tile_prod[k] * carry_r.  The fix-up rebuilds a and b of the leading tiles
// with the scan's own (rounded) arithmetic, runs the recurrence from that
// corrected fp32 state and rewrites those tiles' outputs -- so the result is
// the whole-sequence scan up to fp32 association, with no second rounding of
// already-rounded outputs.
//
// The gated form rewrites a tile while the product of a before it exceeds
// kFixTau = 2^-24 on some channel of the tile (then the correction entering it
// exceeds 2^-24 * |carry| there); with decays in (0, 1) only the leading
// ~log(2^-24)/log(mean a) tokens of a slice are touched.  The rule does not
// depend on the carry, so the local scan (need_sp_local_scan) decides it per
// tile, lists those tiles (args->sp_list) and leaves their rounded updates b
// in their output rows.  The scan kernel in fix-up mode (TMA tiles, the row
// warps' two-phase scan) then rewrites the listed tiles from their decay
// logits and those b, its resident CTAs striding over the list, each
// composing the carry from the gathered maps.  The affine form uses
// fixup_kernel: one warp per tile walks the rows in order, rewriting every
// tile whose correction is non-zero (its decays may exceed 1).
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
    const void* in[2];  // decay (full or per row), update
    int64_t isb[3], ish[3], ist[3];
    void* out;
    int64_t osb, osh, ost;
    const uint8_t* seg;
    int64_t sgb, sgt;
    const float* tile_prod;
    const float* tile_carry;
    const float* all_summary;
    float* h_final;
    float* summary;
};

// Channels per lane of a fix-up warp (a warp covers 32 x kFixLane channels).
#ifndef NEED_FIX_LANE
#define NEED_FIX_LANE 4
#endif
constexpr int kFixLane = NEED_FIX_LANE;
constexpr int kFixChannels = 32 * kFixLane;
constexpr int kFixPairs = kFixLane / 2;

// One row's inputs for one lane (kFixLane channels), loaded ahead of their use.
template <typename TS, typename TD>
struct RowIn {
    typename Ops<TS>::P u[kFixPairs];  // update
    typename Ops<TD>::P d[kFixPairs];  // decay per channel
    float dr;                          // decay per row
    bool reset;
};

// kFixLane consecutive elements as packed pairs
template <typename T>
__device__ __forceinline__ void ldp(const T* p, typename Ops<T>::P (&v)[kFixPairs]) {
    using P = typename Ops<T>::P;
#pragma unroll
    for (int i = 0; i < kFixPairs; ++i) v[i] = reinterpret_cast<const P*>(p)[i];
}

// The affine form's fix-up.  TS: dtype of the update stream and out; TD:
// dtype of the decay.
template <typename TS, typename TD>
__global__ void __launch_bounds__(128) fixup_kernel(const FixParams p) {
    using O = Ops<TS>;
    using PS = typename O::P;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile = blockIdx.x * 4 + warp;
    if (tile >= p.ntiles) return;
    const int chunk = tile / p.nchains;
    const int chain = tile - chunk * p.nchains;
    const int seq = chain / p.ncb;
    const int cblk = chain - seq * p.ncb;
    const int bi = seq / p.nh, hi = seq - bi * p.nh;
    const int c = cblk * kFixChannels + lane * kFixLane;
    const bool active = c < p.C;

    float carry[kFixLane], h[kFixLane];
    bool need = false;
#pragma unroll
    for (int e = 0; e < kFixLane; ++e) {
        carry[e] = 0.0f;
        h[e] = 0.0f;
    }
    if (active) {
        const size_t nsc = size_t(p.nb) * p.nh * p.C;
        for (int j = 0; j < p.rank; ++j) {
            const float2* sj = reinterpret_cast<const float2*>(p.all_summary) + j * nsc + size_t(seq) * p.C + c;
#pragma unroll
            for (int e = 0; e < kFixLane; ++e) {
                const float2 m = sj[e];
                carry[e] = fmaf(m.x, carry[e], m.y);
            }
        }
        const size_t ti = (size_t(seq) * p.nchunks + chunk) * p.C + c;
#pragma unroll
        for (int e = 0; e < kFixLane; ++e) {
            const float corr = p.tile_prod[ti + e] * carry[e];
            h[e] = p.tile_carry[ti + e] + corr;
            need |= corr != 0.0f;  // affine decays may exceed 1: any correction counts
        }
    }
    // slice summary / final state: the chunk-0 warp of each chain
    if (chunk == 0 && active) {
        const float2* mine = reinterpret_cast<const float2*>(p.all_summary) +
                             size_t(p.rank) * p.nb * p.nh * p.C + size_t(seq) * p.C + c;
#pragma unroll
        for (int e = 0; e < kFixLane; ++e) {
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
    // A warp walks its tile's rows in order; the loads of the next D rows are
    // in flight while a row is computed (the rows' inputs do not depend on h).
#ifndef NEED_FIX_DEPTH
#define NEED_FIX_DEPTH 8
#endif
    constexpr int D = Ops<TS>::BYTES == 2 ? NEED_FIX_DEPTH : (NEED_FIX_DEPTH + 1) / 2;
    RowIn<TS, TD> buf[D];
    auto load_row = [&](int r, RowIn<TS, TD>& in) {
        const int64_t t = t0 + r;
        in.reset = p.seg != nullptr && p.seg[bi * p.sgb + t * p.sgt] != 0;
        if (p.rowdec) in.dr = to_f(reinterpret_cast<const TD*>(p.in[0])[bi * p.isb[0] + hi * p.ish[0] + t * p.ist[0]]);
        else ldp<TD>(reinterpret_cast<const TD*>(p.in[0]) + bi * p.isb[0] + hi * p.ish[0] + t * p.ist[0] + c, in.d);
        ldp<TS>(reinterpret_cast<const TS*>(p.in[1]) + bi * p.isb[1] + hi * p.ish[1] + t * p.ist[1] + c, in.u);
    };
    auto compute_row = [&](int r, const RowIn<TS, TD>& in) {
        PS o[kFixPairs];
#pragma unroll
        for (int i = 0; i < kFixPairs; ++i) {
            float2 a = p.rowdec ? make_float2(in.dr, in.dr) : Ops<TD>::unpack(in.d[i]);
            if (in.reset) a = make_float2(0.0f, 0.0f);
            const float2 b = O::unpack(in.u[i]);
            h[2 * i] = fmaf(a.x, h[2 * i], b.x);
            h[2 * i + 1] = fmaf(a.y, h[2 * i + 1], b.y);
            o[i] = O::pack(h[2 * i], h[2 * i + 1]);
        }
        PS* dst = reinterpret_cast<PS*>(orow + (int64_t)(t0 + r) * p.ost);
#pragma unroll
        for (int i = 0; i < kFixPairs; ++i) dst[i] = o[i];
    };
#pragma unroll
    for (int j = 0; j < D; ++j)
        if (j < nrows) load_row(j, buf[j]);
    for (int r0 = 0; r0 < nrows; r0 += D) {
#pragma unroll
        for (int j = 0; j < D; ++j) {
            const int r = r0 + j;
            if (r < nrows) {
                compute_row(r, buf[j]);
                if (r + D < nrows) load_row(r + D, buf[j]);
            }
        }
    }
}

}  // namespace

namespace need {
int gated_fixup_launch(const need_scan_args* a, const float* all_summary, int32_t rank, cudaStream_t stream);
}

extern "C" int need_sp_fixup(const need_scan_args* a, const float* all_summary, int32_t nranks, int32_t rank,
                             need_stream_t stream) {
    if (a == nullptr || all_summary == nullptr) return fail(NEED_ERR_INVALID, "null argument");
    if (a->form != NEED_FORM_GATED && a->form != NEED_FORM_AFFINE)
        return fail(NEED_ERR_UNSUPPORTED, "sequence-parallel fix-up takes the GATED or AFFINE form");
    if (nranks < 1 || rank < 0 || rank >= nranks) return fail(NEED_ERR_INVALID, "rank %d of %d", rank, nranks);
    if (a->nb < 1 || a->nh < 1 || a->T < 1 || a->C < 1) return fail(NEED_ERR_INVALID, "bad sizes");
    if (a->C % 8 != 0) return fail(NEED_ERR_UNSUPPORTED, "C must be a multiple of 8");
    if (a->tile_prod == nullptr || a->tile_carry == nullptr)
        return fail(NEED_ERR_INVALID, "tile_prod / tile_carry are null (request them from the local scan)");
    if (!aligned16(a->out)) return fail(NEED_ERR_UNSUPPORTED, "out is not 16-byte aligned");
    const bool gated = a->form == NEED_FORM_GATED;
    const int rd = gated ? 0 : (a->decay_per_row ? 1 : 0);
    const int ddt = gated ? a->dtype : a->decay_dtype;
    const int64_t L = need_scan_chunk_len(a->form, a->dtype, ddt, rd);
    if (L <= 0) return fail(NEED_ERR_UNSUPPORTED, "no kernel for this dtype combination");
    const int nin = gated ? 3 : 2;
    for (int k = 0; k < nin; ++k) {
        if (a->in[k].ptr == nullptr) return fail(NEED_ERR_INVALID, "in[%d] is null", k);
        if (!(k == 0 && rd) && !aligned16(a->in[k].ptr)) return fail(NEED_ERR_UNSUPPORTED, "in[%d] is not 16-byte aligned", k);
    }
    if (rank == 0) return ok();  // no carry enters the first slice

    if (gated) {
        // The gated form re-scans the tiles its deferring local scan listed in
        // a->sp_list, with the scan kernel itself (fix-up mode), in one launch.
        if (int rc = gated_fixup_launch(a, all_summary, rank, stream)) return rc;
        return ok();
    }

    FixParams p{};
    p.form = a->form;
    p.rowdec = rd;
    p.nb = int32_t(a->nb);
    p.nh = int32_t(a->nh);
    p.T = int32_t(a->T);
    p.C = int32_t(a->C);
    p.L = int32_t(L);
    p.ncb = int32_t((a->C + kFixChannels - 1) / kFixChannels);
    p.nchains = p.nb * p.nh * p.ncb;
    p.nchunks = int32_t((a->T + L - 1) / L);
    p.ntiles = p.nchains * p.nchunks;
    p.nranks = nranks;
    p.rank = rank;
    for (int k = 0; k < nin; ++k) {
        p.in[k] = a->in[k].ptr;
        p.isb[k] = a->in[k].stride_b;
        p.ish[k] = a->in[k].stride_h;
        p.ist[k] = a->in[k].stride_t;
    }
    p.out = a->out;
    p.osb = a->out_stride_b;
    p.osh = a->out_stride_h;
    p.ost = a->out_stride_t;
    p.seg = a->seg_start;
    p.sgb = a->seg_stride_b;
    p.sgt = a->seg_stride_t;
    p.tile_prod = a->tile_prod;
    p.tile_carry = a->tile_carry;
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
