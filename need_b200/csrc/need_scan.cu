// need_scan.cu -- C ABI of the chunked-scan kernels (need_scan.h): argument
// validation, TMA descriptor encoding, tile planning and launch.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <climits>
#include <mutex>

#include "host_common.h"
#include "need_scan.h"
#include "scan_kernel.cuh"

using namespace need;
using bf16 = __nv_bfloat16;
using f16 = __half;

namespace {

// ------------------------------------------------------------------ plans
// One instantiation of scan_kernel per (form, stream dtype, decay dtype,
// row-broadcast decay).  Tile lengths keep each CTA's staged tile near 96 KB
// so two CTAs fit an SM's 228 KB of shared memory.
// Tile shape of the 16-bit gated scan (tokens per tile, warps per CTA,
// channels per tile): 128 x 128 was the fastest of the shapes measured on
// B200 for the B=16, T=4096, C=1024 prefill (128 chains of 32 chunks).
#ifndef NEED_GATED16_L
#define NEED_GATED16_L 128
#endif
#ifndef NEED_GATED16_NW
#define NEED_GATED16_NW 8
#endif
#ifndef NEED_GATED16_CB
#define NEED_GATED16_CB 128
#endif
template <typename T>
using GatedCfg = ScanCfg<FORM_GATED, T, T, false, sizeof(T) == 2 ? NEED_GATED16_L : 32,
                         sizeof(T) == 2 ? NEED_GATED16_NW : 4, sizeof(T) == 2 ? NEED_GATED16_CB : 256>;
// Tile shape of the 16-bit SSD scan: 64 tokens x 64 channels x 4 warps (up to 4
// CTAs per SM) measured fastest of 9 shapes at NEED's model shape (B=8, T=2048,
// C=832: 47.5 us against 56.2 us for 64 x 128 x 8 warps) and at B=16, T=4096,
// C=1024 (190 against 213.7 us).
#ifndef NEED_SSD16_L
#define NEED_SSD16_L 64
#endif
#ifndef NEED_SSD16_NW
#define NEED_SSD16_NW 4
#endif
#ifndef NEED_SSD16_CB
#define NEED_SSD16_CB 64
#endif
template <typename T>
using SsdCfg = ScanCfg<FORM_SSD, T, T, false, sizeof(T) == 2 ? NEED_SSD16_L : 16, sizeof(T) == 2 ? NEED_SSD16_NW : 4,
                       sizeof(T) == 2 ? NEED_SSD16_CB : 256>;
// The 16-bit SSD scan with the block's conv + SiLU folded into its tile loads.
template <typename T, int KC>
using SsdConvCfg = ScanCfg<FORM_SSD, T, T, false, NEED_SSD16_L, NEED_SSD16_NW, NEED_SSD16_CB, KC>;
static_assert(SsdConvCfg<bf16, 3>::L == SsdCfg<bf16>::L && SsdConvCfg<bf16, 3>::CBW == SsdCfg<bf16>::CBW &&
                  SsdConvCfg<bf16, 3>::R == SsdCfg<bf16>::R,
              "the folded-conv scan shares the SSD plan's tiles, tensor maps and workspace");

#ifndef NEED_AFF16_L
#define NEED_AFF16_L 128
#endif
#ifndef NEED_AFF16_NW
#define NEED_AFF16_NW 4
#endif
#ifndef NEED_AFF16_CB
#define NEED_AFF16_CB 128
#endif
template <typename TS, typename TD, bool RD>
struct AffL {
    static constexpr bool B16 = !RD && sizeof(TS) == 2 && sizeof(TD) == 2;  // 16-bit decay and update streams
    static constexpr int L = RD ? (sizeof(TS) == 2 ? 64 : 32) : (B16 ? NEED_AFF16_L : 32);
    static constexpr int NW = B16 ? NEED_AFF16_NW : 8;
    static constexpr int CB = B16 ? NEED_AFF16_CB : 256;
};
template <typename TS, typename TD, bool RD>
using AffCfg = ScanCfg<FORM_AFFINE, TS, TD, RD, AffL<TS, TD, RD>::L, AffL<TS, TD, RD>::NW, AffL<TS, TD, RD>::CB>;

template <typename TS, typename TD, bool RD>
struct RetL {
    static constexpr bool SMALL = !RD && sizeof(TS) == 4;
    static constexpr int L = RD ? (sizeof(TS) == 2 ? 64 : 32) : (SMALL ? 16 : 32);
    static constexpr int NW = SMALL ? 4 : 8;
};
template <typename TS, typename TD, bool RD>
using RetCfg = ScanCfg<FORM_RETENTION, TS, TD, RD, RetL<TS, TD, RD>::L, RetL<TS, TD, RD>::NW>;

struct Plan {
    int L = 0, R = 0, CB = 0, nin = 0, in0 = 0;  // tokens, rows per warp, channels per tile
    bool dstream = false, split = false;
    int (*launch)(const ScanParams&, cudaStream_t) = nullptr;
    int (*launch_fix)(const ScanParams&, cudaStream_t) = nullptr;   // gated form only
    int (*launch_defer)(const ScanParams&, cudaStream_t) = nullptr; // gated form only
    int (*launch_rev)(const ScanParams&, cudaStream_t) = nullptr;   // affine form only
};

template <class K>
int launch_cfg(const ScanParams& prm, cudaStream_t s) {
    static std::atomic<uint64_t> smem_done{0};
    cudaError_t e = ensure_smem(scan_kernel<K>, K::SMEM, smem_done);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(scan_kernel)");
    scan_kernel<K><<<prm.ntiles, K::NT, K::SMEM, s>>>(prm);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "scan_kernel launch");
    return NEED_OK;
}

// The local scan of a sequence-parallel slice after the first (DEFER), one tile per CTA.
template <class K>
int launch_defer_cfg(const ScanParams& prm, cudaStream_t s) {
    static std::atomic<uint64_t> smem_done{0};
    cudaError_t e = ensure_smem(scan_kernel<K, false, false, true>, K::SMEM, smem_done);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(scan_kernel, deferred)");
    scan_kernel<K, false, false, true><<<prm.ntiles, K::NT, K::SMEM, s>>>(prm);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "scan_kernel launch (deferred)");
    return NEED_OK;
}

// The sequence-parallel fix-up: as many CTAs as fit on the device at once
// (occupancy x SMs, found once per device), striding over the tiles to rewrite.
template <class K>
int launch_fix_cfg(const ScanParams& prm, cudaStream_t s) {
    static std::atomic<uint64_t> smem_done{0};
    static std::atomic<int> resident[kMaxDevices];
    cudaError_t e = ensure_smem(scan_kernel<K, true>, K::SMEM, smem_done);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(scan_kernel, fix-up)");
    int dev = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) return fail(NEED_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
    int ctas = resident[dev].load(std::memory_order_relaxed);
    if (ctas == 0) {
        int per_sm = 0, sms = 0;
        if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, scan_kernel<K, true>, K::NT, K::SMEM)) !=
            cudaSuccess)
            return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
        if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
            return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
        ctas = std::max(1, per_sm) * std::max(1, sms);
        resident[dev].store(ctas, std::memory_order_relaxed);
    }
    scan_kernel<K, true><<<std::min(ctas, prm.ntiles), K::NT, K::SMEM, s>>>(prm);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "scan_kernel launch (fix-up)");
    return NEED_OK;
}

// The reversed-time scan (the backward's adjoint recurrence), one tile per CTA.
template <class K>
int launch_rev_cfg(const ScanParams& prm, cudaStream_t s) {
    static std::atomic<uint64_t> smem_done{0};
    cudaError_t e = ensure_smem(scan_kernel<K, false, true>, K::SMEM, smem_done);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(scan_kernel, reversed)");
    scan_kernel<K, false, true><<<prm.ntiles, K::NT, K::SMEM, s>>>(prm);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "scan_kernel launch (reversed)");
    return NEED_OK;
}

template <class K>
Plan plan_of() {
    Plan p;
    p.L = K::L;
    p.R = K::R;
    p.CB = K::CBW;
    p.nin = K::NIN;
    p.in0 = K::IN0;
    p.dstream = K::HAS_DSTREAM;
    p.split = K::SPLIT;
    p.launch = &launch_cfg<K>;
    if constexpr (K::FORM == FORM_GATED) {
        p.launch_fix = &launch_fix_cfg<K>;
        p.launch_defer = &launch_defer_cfg<K>;
    }
    if constexpr (K::FORM == FORM_AFFINE) p.launch_rev = &launch_rev_cfg<K>;
    return p;
}

template <template <typename, typename, bool> class CFG>
bool plan_decay(int dt, int ddt, int rd, Plan* out) {
    // decay dtype either equals the stream dtype or is fp32
    if (dt == NEED_F32 && ddt == NEED_F32) *out = rd ? plan_of<CFG<float, float, true>>() : plan_of<CFG<float, float, false>>();
    else if (dt == NEED_BF16 && ddt == NEED_BF16) *out = rd ? plan_of<CFG<bf16, bf16, true>>() : plan_of<CFG<bf16, bf16, false>>();
    else if (dt == NEED_BF16 && ddt == NEED_F32) *out = rd ? plan_of<CFG<bf16, float, true>>() : plan_of<CFG<bf16, float, false>>();
    else if (dt == NEED_F16 && ddt == NEED_F16) *out = rd ? plan_of<CFG<f16, f16, true>>() : plan_of<CFG<f16, f16, false>>();
    else if (dt == NEED_F16 && ddt == NEED_F32) *out = rd ? plan_of<CFG<f16, float, true>>() : plan_of<CFG<f16, float, false>>();
    else return false;
    return true;
}

bool select_plan(int form, int dt, int ddt, int rd, Plan* out) {
    if (!dtype_ok(dt)) return false;
    switch (form) {
        case NEED_FORM_GATED:
            if (dt == NEED_F32) *out = plan_of<GatedCfg<float>>();
            else if (dt == NEED_BF16) *out = plan_of<GatedCfg<bf16>>();
            else *out = plan_of<GatedCfg<f16>>();
            return true;
        case NEED_FORM_SSD:
            if (dt == NEED_F32) *out = plan_of<SsdCfg<float>>();
            else if (dt == NEED_BF16) *out = plan_of<SsdCfg<bf16>>();
            else *out = plan_of<SsdCfg<f16>>();
            return true;
        case NEED_FORM_AFFINE:
            return plan_decay<AffCfg>(dt, ddt, rd ? 1 : 0, out);
        case NEED_FORM_RETENTION:
            return plan_decay<RetCfg>(dt, ddt, rd ? 1 : 0, out);
        default:
            return false;
    }
}

int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Look-back polls before a wait gives up, for the launches that follow; 0 =
// the default kLookbackPolls.  Set only by need_test_set_lookback_polls.
std::atomic<uint32_t> g_lookback_polls{0};


struct Geometry {
    int64_t ncb, nchains, nchunks, ntiles;
};

Geometry geometry(const Plan& pl, int64_t nb, int64_t nh, int64_t T, int64_t C) {
    Geometry g;
    g.ncb = cdiv(C, pl.CB);
    g.nchains = nb * nh * g.ncb;
    g.nchunks = cdiv(T, pl.L);
    g.ntiles = g.nchains * g.nchunks;
    return g;
}

size_t ws_bytes(const Plan& pl, int64_t ntiles) {
    const size_t hdr = WS_HDR_WORDS * 4;
    return hdr + size_t(ntiles) * size_t(pl.CB) * sizeof(ulonglong2) * 2;  // tagged AGG and INCL records
}

// ------------------------------------------------------------------ TMA descriptors
int encode_view(CUtensorMap* tm, const need_view& v, int dt, int64_t nb, int64_t nh, int64_t T, int64_t C,
                int box_c, int box_rows, int which) {
    if (v.ptr == nullptr) return fail(NEED_ERR_INVALID, "in[%d] is null", which);
    if (!aligned16(v.ptr)) return fail(NEED_ERR_UNSUPPORTED, "in[%d] is not 16-byte aligned", which);
    const int64_t es = dtype_bytes(dt);
    const int64_t sizes[3] = {T, nh, nb};
    const int64_t strides[3] = {v.stride_t, v.stride_h, v.stride_b};
    cuuint64_t gs[3];
    int64_t prev = ((C * es + 15) / 16) * 16;  // packed stride for size-1 dims
    for (int i = 0; i < 3; ++i) {
        if (sizes[i] == 1) {
            gs[i] = static_cast<cuuint64_t>(prev);
        } else {
            const int64_t b = strides[i] * es;
            if (strides[i] <= 0 || (b % 16) != 0 || b >= (int64_t(1) << 40))
                return fail(NEED_ERR_UNSUPPORTED,
                            "in[%d]: stride %lld (dim %d) must be positive and a multiple of 16 bytes", which,
                            static_cast<long long>(strides[i]), i);
            gs[i] = static_cast<cuuint64_t>(b);
        }
        prev = static_cast<int64_t>(gs[i]) * sizes[i];
    }
    const cuuint64_t dims[4] = {cuuint64_t(C), cuuint64_t(T), cuuint64_t(nh), cuuint64_t(nb)};
    const cuuint32_t box[4] = {cuuint32_t(box_c), cuuint32_t(box_rows), 1, 1};  // one warp's rows
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUtensorMapDataType ty = dt == NEED_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : dt == NEED_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                     : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    auto fn = encode_fn();
    if (fn == nullptr) return fail(NEED_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    const CUresult r = fn(tm, ty, 4, const_cast<void*>(v.ptr), dims, gs, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(NEED_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled(in[%d]) failed: %d", which, int(r));
    return NEED_OK;
}

int check_sizes(const need_scan_args* a) {
    if (a->nb < 1 || a->nh < 1 || a->T < 1 || a->C < 1)
        return fail(NEED_ERR_INVALID, "sizes must be >= 1 (nb=%lld nh=%lld T=%lld C=%lld)", (long long)a->nb,
                    (long long)a->nh, (long long)a->T, (long long)a->C);
    if (a->T > INT32_MAX / 2 || a->C > INT32_MAX / 2 || a->nb * a->nh > INT32_MAX / 2)
        return fail(NEED_ERR_UNSUPPORTED, "sizes exceed the 32-bit tile index range");
    return NEED_OK;
}

// Validates `a` and fills the kernel parameters.
// rev: the backward's reversed scan -- a streamed decay (in[0]) is viewed from
// row 1 with T-1 rows, so row t reads a_{t+1} and row T-1 reads the zero fill.
int prepare(const need_scan_args* a, int expect_form, Plan* pl, ScanParams* P, bool rev = false) {
    if (a == nullptr) return fail(NEED_ERR_INVALID, "args is null");
    if (a->form != expect_form) return fail(NEED_ERR_INVALID, "args->form %d does not match the entry point", a->form);
    if (int rc = check_sizes(a)) return rc;
    const bool rowdec_form = a->form == NEED_FORM_AFFINE || a->form == NEED_FORM_RETENTION;
    const int ddt = rowdec_form ? a->decay_dtype : a->dtype;
    const int rd = rowdec_form ? (a->decay_per_row ? 1 : 0) : 0;
    if (!select_plan(a->form, a->dtype, ddt, rd, pl))
        return fail(NEED_ERR_UNSUPPORTED, "no kernel for form %d dtype %d decay dtype %d", a->form, a->dtype, ddt);
    const Geometry g = geometry(*pl, a->nb, a->nh, a->T, a->C);
    if (g.ntiles > INT32_MAX) return fail(NEED_ERR_UNSUPPORTED, "too many tiles (%lld)", (long long)g.ntiles);
    const int group = pl->split ? 4 : 8;
    if (a->C % group != 0)
        return fail(NEED_ERR_UNSUPPORTED, "C=%lld must be a multiple of %d for this dtype", (long long)a->C, group);

    if (int rc = ensure_context()) return rc;
    memset(P, 0, sizeof(*P));
    for (int k = 0; k < pl->nin; ++k) {
        const int dt = (pl->dstream && k == 0) ? ddt : a->dtype;
        need_view view = a->in[pl->in0 + k];
        int64_t rows = a->T;
        if (rev && pl->dstream && k == 0) {
            view.ptr = static_cast<const unsigned char*>(view.ptr) + view.stride_t * dtype_bytes(dt);
            rows = a->T - 1;
        }
        if (int rc = encode_view(&P->tm[k], view, dt, a->nb, a->nh, rows, a->C, pl->CB, pl->R, pl->in0 + k))
            return rc;
    }
    if (rowdec_form && rd) {
        if (a->in[0].ptr == nullptr) return fail(NEED_ERR_INVALID, "in[0] (row decay) is null");
        P->rowdec = a->in[0].ptr;
        P->dsb = a->in[0].stride_b;
        P->dsh = a->in[0].stride_h;
        P->dst = a->in[0].stride_t;
    }
    if (a->out == nullptr) return fail(NEED_ERR_INVALID, "out is null");
    if (!aligned16(a->out)) return fail(NEED_ERR_UNSUPPORTED, "out is not 16-byte aligned");
    const int64_t ostr[3] = {a->out_stride_t, a->out_stride_h, a->out_stride_b};
    const int64_t osz[3] = {a->T, a->nh, a->nb};
    for (int i = 0; i < 3; ++i)
        if (osz[i] > 1 && (ostr[i] <= 0 || ostr[i] % group != 0))
            return fail(NEED_ERR_UNSUPPORTED, "out stride %lld must be a positive multiple of %d elements",
                        (long long)ostr[i], group);
    if (a->form == NEED_FORM_SSD && a->d_skip == nullptr) return fail(NEED_ERR_INVALID, "d_skip is null");
    if (a->workspace == nullptr) return fail(NEED_ERR_WORKSPACE, "workspace is null");
    if (!aligned16(a->workspace)) return fail(NEED_ERR_WORKSPACE, "workspace is not 16-byte aligned");
    const size_t need = ws_bytes(*pl, g.ntiles);
    if (a->workspace_bytes < need)
        return fail(NEED_ERR_WORKSPACE, "workspace has %zu bytes, needs %zu", a->workspace_bytes, need);

    P->nb = int32_t(a->nb);
    P->nh = int32_t(a->nh);
    P->T = int32_t(a->T);
    P->C = int32_t(a->C);
    P->ncb = int32_t(g.ncb);
    P->nchains = int32_t(g.nchains);
    P->nchunks = int32_t(g.nchunks);
    P->ntiles = int32_t(g.ntiles);
    P->out = a->out;
    P->osb = a->out_stride_b;
    P->osh = a->out_stride_h;
    P->ost = a->out_stride_t;
    P->dskip = a->d_skip;
    // need_kernels.py:331: the Python floats enter fp32 arithmetic as fp32
    P->dt_min = static_cast<float>(a->dt_min);
    P->dt_scale = static_cast<float>(a->dt_max - a->dt_min);
    P->h0 = a->h0;
    P->h_final = a->h_final;
    P->seg = a->seg_start;
    P->sgb = a->seg_stride_b;
    P->sgt = a->seg_stride_t;
    P->summary = a->summary;
    P->tile_prod = a->tile_prod;
    P->tile_carry = a->tile_carry;
    unsigned char* ws = static_cast<unsigned char*>(a->workspace);
    P->hdr = reinterpret_cast<uint32_t*>(ws);
    const uint32_t polls = g_lookback_polls.load(std::memory_order_relaxed);
    P->lb_polls = polls != 0 ? polls : kLookbackPolls;
    P->agg = reinterpret_cast<ulonglong2*>(ws + WS_HDR_WORDS * 4);
    P->incl = P->agg + size_t(g.ntiles) * pl->CB;
    return NEED_OK;
}

int run(const need_scan_args* a, int form, cudaStream_t s) {
    Plan pl;
    ScanParams P;
    if (int rc = prepare(a, form, &pl, &P)) return rc;
    if (int rc = pl.launch(P, s)) return rc;
    return ok();
}

// The words of a slice's sequence-parallel list: the count (4 words, 16-byte
// aligned entries after it) and up to ntiles tile ids.
constexpr int64_t kSpListHead = 4;

// Points P's sequence-parallel list at args->sp_list (checked for its size).
int sp_list_of(const need_scan_args* a, ScanParams* P) {
    if (a->sp_list == nullptr) return fail(NEED_ERR_INVALID, "sp_list is null (need_sp_list_size words)");
    if (reinterpret_cast<uintptr_t>(a->sp_list) % 4 != 0) return fail(NEED_ERR_INVALID, "sp_list is not 4-byte aligned");
    const uint64_t need = uint64_t(kSpListHead) + uint64_t(P->ntiles);
    if (a->sp_list_words < need)
        return fail(NEED_ERR_WORKSPACE, "sp_list holds %llu words, needs %llu (need_sp_list_size)",
                    (unsigned long long)a->sp_list_words, (unsigned long long)need);
    P->sp_count = a->sp_list;
    P->sp_list = a->sp_list + kSpListHead;
    return NEED_OK;
}

}  // namespace

namespace need {
// The gated scan kernel in fix-up mode over the slice described by `a`: it
// rewrites the tiles that the deferring local scan listed in a->sp_list (and
// whose rounded updates b it left in their output rows), entering each from the local scan's tile_prod / tile_carry and
// the carry it composes from all_summary [nranks][nb*nh][C] (ranks < rank);
// the chain's first tile also corrects h_final and summary.  Writes only the
// rewritten tiles' outputs.
int gated_fixup_launch(const need_scan_args* a, const float* all_summary, int32_t rank, cudaStream_t stream) {
    Plan pl;
    ScanParams P;
    if (int rc = prepare(a, NEED_FORM_GATED, &pl, &P)) return rc;
    if (pl.launch_fix == nullptr) return fail(NEED_ERR_UNSUPPORTED, "no fix-up kernel for dtype %d", a->dtype);
    if (int rc = sp_list_of(a, &P)) return rc;
    // the rounded updates b the deferring local scan left in the listed tiles' output rows
    const need_view ov{a->out, a->out_stride_b, a->out_stride_h, a->out_stride_t};
    if (int rc = encode_view(&P.tm[3], ov, a->dtype, a->nb, a->nh, a->T, a->C, pl.CB, pl.R, 3)) return rc;
    P.fix_tile_prod = a->tile_prod;
    P.fix_tile_carry = a->tile_carry;
    P.fix_all_summary = reinterpret_cast<const float2*>(all_summary);
    P.fix_rank = rank;
    P.tile_prod = nullptr;
    P.tile_carry = nullptr;
    P.h0 = nullptr;
    return pl.launch_fix(P, stream);
}
}  // namespace need

// ------------------------------------------------------------------ exported
extern "C" {

int need_abi_version(void) { return NEED_SCAN_ABI_VERSION; }

const char* need_last_error(void) { return last_error_slot().c_str(); }

int64_t need_scan_chunk_len(int32_t form, int32_t dtype, int32_t decay_dtype, int32_t decay_per_row) {
    Plan pl;
    const bool rf = form == NEED_FORM_AFFINE || form == NEED_FORM_RETENTION;
    if (!select_plan(form, dtype, rf ? decay_dtype : dtype, rf ? decay_per_row : 0, &pl)) return -1;
    return pl.L;
}

size_t need_scan_workspace_size(int32_t form, int32_t dtype, int32_t decay_dtype, int32_t decay_per_row, int64_t nb,
                                int64_t nh, int64_t T, int64_t C) {
    Plan pl;
    const bool rf = form == NEED_FORM_AFFINE || form == NEED_FORM_RETENTION;
    if (!select_plan(form, dtype, rf ? decay_dtype : dtype, rf ? decay_per_row : 0, &pl)) return 0;
    if (nb < 1 || nh < 1 || T < 1 || C < 1) return ws_bytes(pl, 0);
    return ws_bytes(pl, geometry(pl, nb, nh, T, C).ntiles);
}

void need_test_set_lookback_polls(uint32_t polls) { g_lookback_polls.store(polls, std::memory_order_relaxed); }

int need_workspace_error(void* workspace, uint32_t* error_out, need_stream_t stream) {
    if (workspace == nullptr || error_out == nullptr) return fail(NEED_ERR_INVALID, "null argument");
    uint32_t* word = static_cast<uint32_t*>(workspace) + WS_ERROR;
    cudaError_t e = cudaMemcpyAsync(error_out, word, 4, cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(word, 0, 4, stream);
    if (e != cudaSuccess) return cuda_fail(e, "need_workspace_error");
    return ok();
}

int need_affine_recurrence_scan(const need_scan_args* args, need_stream_t stream) {
    return run(args, NEED_FORM_AFFINE, stream);
}

int need_affine_recurrence_scan_backward(const need_scan_args* args, need_stream_t stream) {
    if (args == nullptr) return fail(NEED_ERR_INVALID, "args is null");
    if (args->seg_start != nullptr || args->h0 != nullptr || args->summary != nullptr ||
        args->tile_prod != nullptr || args->tile_carry != nullptr)
        return fail(NEED_ERR_INVALID, "the backward scan takes no seg_start, h0, summary or tile records");
    if (args->T < 2) return fail(NEED_ERR_INVALID, "the backward scan needs T >= 2 (for T = 1 the gradient is g)");
    Plan pl;
    ScanParams P;
    if (int rc = prepare(args, NEED_FORM_AFFINE, &pl, &P, true)) return rc;
    if (pl.launch_rev == nullptr) return fail(NEED_ERR_UNSUPPORTED, "no reversed scan for this dtype combination");
    if (int rc = pl.launch_rev(P, stream)) return rc;
    return ok();
}

int need_ssd_scan(const need_scan_args* args, need_stream_t stream) { return run(args, NEED_FORM_SSD, stream); }

int need_ssd_scan_rms_norm(const need_scan_args* args, const void* norm_weight, int32_t weight_dtype, double eps,
                           need_stream_t stream) {
    if (args == nullptr) return fail(NEED_ERR_INVALID, "args is null");
    if (norm_weight == nullptr) return fail(NEED_ERR_INVALID, "norm_weight is null");
    if (weight_dtype != NEED_F32 && weight_dtype != args->dtype)
        return fail(NEED_ERR_UNSUPPORTED, "norm weight dtype %d must be fp32 or the stream dtype %d", weight_dtype,
                    args->dtype);
    if (!(eps >= 0.0)) return fail(NEED_ERR_INVALID, "eps must be >= 0");
    if (args->nh != 1) return fail(NEED_ERR_UNSUPPORTED, "the RMSNorm epilogue takes nh == 1");
    Plan pl;
    ScanParams P;
    if (int rc = prepare(args, NEED_FORM_SSD, &pl, &P)) return rc;
    if (int rc = pl.launch(P, stream)) return rc;
    // the normalisation over the rows just written, in place, while they are in L2
    if (int rc = rms_norm_rows(args->dtype, args->out, args->out_stride_b, args->out_stride_t, args->out,
                               args->out_stride_b, args->out_stride_t, args->nb, args->T, args->C, norm_weight,
                               weight_dtype, eps, stream))
        return rc;
    return ok();
}

int need_ssd_conv_scan(const need_scan_args* args, const need_ssd_conv* conv, const void* norm_weight,
                       int32_t weight_dtype, double eps, need_stream_t stream) {
    if (args == nullptr || conv == nullptr) return fail(NEED_ERR_INVALID, "null argument");
    if (args->dtype != NEED_BF16 && args->dtype != NEED_F16)
        return fail(NEED_ERR_UNSUPPORTED, "the folded conv takes bf16 or f16 data");
    if (conv->K < 1 || conv->K > kConvHalo + 1)
        return fail(NEED_ERR_UNSUPPORTED, "K=%d taps (1..%d supported)", conv->K, kConvHalo + 1);
    if (conv->weight == nullptr) return fail(NEED_ERR_INVALID, "conv weight is null");
    if (args->nh != 1) return fail(NEED_ERR_UNSUPPORTED, "the folded conv takes nh == 1");
    if (norm_weight != nullptr) {
        if (weight_dtype != NEED_F32 && weight_dtype != args->dtype)
            return fail(NEED_ERR_UNSUPPORTED, "norm weight dtype %d must be fp32 or the stream dtype %d",
                        weight_dtype, args->dtype);
        if (!(eps >= 0.0)) return fail(NEED_ERR_INVALID, "eps must be >= 0");
    }
    Plan pl;
    ScanParams P;
    if (int rc = prepare(args, NEED_FORM_SSD, &pl, &P)) return rc;
    // the raw u rows before each warp's rows: a box of kConvHalo rows of in[2]
    if (int rc = encode_view(&P.tm_halo, args->in[2], args->dtype, args->nb, args->nh, args->T, args->C, pl.CB,
                             kConvHalo, 2))
        return rc;
    P.conv_w = conv->weight;
    P.cwsc = conv->w_stride_c;
    P.cwsk = conv->w_stride_k;
    P.conv_b = conv->bias;
    int rc = NEED_OK;
    const bool b16 = args->dtype == NEED_BF16;
    switch (conv->K) {  // the tap count is compiled in
        case 1: rc = b16 ? launch_cfg<SsdConvCfg<bf16, 1>>(P, stream) : launch_cfg<SsdConvCfg<f16, 1>>(P, stream); break;
        case 2: rc = b16 ? launch_cfg<SsdConvCfg<bf16, 2>>(P, stream) : launch_cfg<SsdConvCfg<f16, 2>>(P, stream); break;
        case 3: rc = b16 ? launch_cfg<SsdConvCfg<bf16, 3>>(P, stream) : launch_cfg<SsdConvCfg<f16, 3>>(P, stream); break;
        default: rc = b16 ? launch_cfg<SsdConvCfg<bf16, 4>>(P, stream) : launch_cfg<SsdConvCfg<f16, 4>>(P, stream); break;
    }
    if (rc) return rc;
    if (norm_weight != nullptr) {
        if (int r2 = rms_norm_rows(args->dtype, args->out, args->out_stride_b, args->out_stride_t, args->out,
                                   args->out_stride_b, args->out_stride_t, args->nb, args->T, args->C, norm_weight,
                                   weight_dtype, eps, stream))
            return r2;
    }
    return ok();
}

int need_recurrent_retention_scan(const need_scan_args* args, need_stream_t stream) {
    return run(args, NEED_FORM_RETENTION, stream);
}

int need_sp_local_scan(const need_scan_args* args, int32_t rank, need_stream_t stream) {
    if (args == nullptr) return fail(NEED_ERR_INVALID, "args is null");
    if (rank < 0) return fail(NEED_ERR_INVALID, "rank %d", rank);
    if (args->summary == nullptr || args->tile_prod == nullptr || args->tile_carry == nullptr)
        return fail(NEED_ERR_INVALID, "the local scan of a slice needs summary, tile_prod and tile_carry");
    Plan pl;
    ScanParams P;
    if (int rc = prepare(args, NEED_FORM_GATED, &pl, &P)) return rc;
    if (rank == 0) {  // every output is written; the list (when given) is left empty
        if (args->sp_list != nullptr) {
            const cudaError_t e = cudaMemsetAsync(args->sp_list, 0, sizeof(uint32_t), stream);
            if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(sequence-parallel list)");
        }
        if (int rc = pl.launch(P, stream)) return rc;
        return ok();
    }
    if (pl.launch_defer == nullptr) return fail(NEED_ERR_UNSUPPORTED, "no deferring scan for dtype %d", args->dtype);
    if (int rc = sp_list_of(args, &P)) return rc;
    const cudaError_t e = cudaMemsetAsync(P.sp_count, 0, sizeof(uint32_t), stream);  // the list starts empty
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(sequence-parallel list)");
    if (int rc = pl.launch_defer(P, stream)) return rc;
    return ok();
}

size_t need_sp_list_size(int32_t dtype, int64_t nb, int64_t nh, int64_t T, int64_t C) {
    Plan pl;
    if (!select_plan(NEED_FORM_GATED, dtype, dtype, 0, &pl)) return 0;
    if (nb < 1 || nh < 1 || T < 1 || C < 1) return size_t(kSpListHead);
    return size_t(kSpListHead + geometry(pl, nb, nh, T, C).ntiles);
}

int need_gated_scan(const need_scan_args* args, need_stream_t stream) { return run(args, NEED_FORM_GATED, stream); }

}  // extern "C"
