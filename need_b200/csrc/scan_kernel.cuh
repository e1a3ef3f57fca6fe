// scan_kernel.cuh -- single-pass chunked scan of h[t] = a[t]*h[t-1] + b[t] for
// sm_100a (B200).
//
// Work decomposition.  A call scans nseq = nb*nh independent sequences of C
// channels over T steps.  A tile is (sequence, CBW-channel block, L-token
// chunk), one CTA per tile, numbered chunk-major by blockIdx.x, so every
// tile's predecessors along T have lower block indices.
//
// Per tile (one CTA: NW row warps and one look-back warp):
//   1. TMA (cp.async.bulk.tensor, no multicast): each row warp loads its own
//      R = L/NW rows of every streamed tensor into shared memory (zero fill
//      past T and C), completing on its own mbarrier.
//   2. Phase 1: a lane owns 8 channels of one or more rows.  Each thread
//      computes a, b for its rows (gate math per form; 16-bit inputs are
//      rounded where the reference's torch path rounds), writes them back in
//      place for phase 2, and reduces its rows to one affine map (A, B):
//      h_out = A*h_in + B.  The row groups of a warp combine their maps by
//      shuffles into in-warp prefixes, and the warp's total map goes to
//      shared memory.
//   3. The look-back warp, from the CTA's start, polls the records of the
//      kLookbackDepth tiles before this one along T (their maps, AGG) and the
//      inclusive state (INCL) of the tile before those, composing them in that
//      fixed order, so results are bit-reproducible; it composes the warps'
//      totals into this tile's map and publishes it the moment they are in,
//      then walks the carry through the warp totals, leaving in shared memory
//      the state entering each warp's rows, and publishes the inclusive
//      state.  Records carry the launch's tag in every 64-bit word, so neither
//      side needs a fence or a flag.  Every wait is bounded; on give-up an
//      error bit is set and the tile continues.
//   4. Phase 2: every thread takes its warp's entering state, applies its
//      in-warp prefix, restarts its rows from there and writes the outputs
//      straight to global memory (16-byte stores).
// HBM traffic is the algorithmic minimum (inputs read once, outputs written
// once) plus 32 bytes of look-back records per channel and tile (normally
// L2-resident).  The same kernel also runs the sequence-parallel fix-up
// (FIX) and the backward's reversed-time scan (REV); see scan_kernel below.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ptx.cuh"

namespace need {

enum { FORM_AFFINE = 0, FORM_GATED = 1, FORM_SSD = 2, FORM_RETENTION = 3 };

// workspace header words (uint32)
// words 0-1: one 64-bit word {launch epoch (high), CTAs started (low)}
// word 3: the error word
enum { WS_LAUNCH = 0, WS_ERROR = 3, WS_HDR_WORDS = 32 };
enum { ERR_LOOKBACK = 1u, ERR_TMA = 2u, ERR_SP_LIST = 4u };

// look-back polls before a wait gives up (each poll is an L2 round trip plus a
// 64 ns sleep: a few seconds at most); need_test_set_lookback_polls lowers it
constexpr uint32_t kLookbackPolls = 1u << 22;
#ifndef NEED_LOOKBACK_DEPTH
#define NEED_LOOKBACK_DEPTH 3
#endif
// Tile maps composed before an inclusive state (at most 31: one lane polls each).
constexpr int kLookbackDepth = NEED_LOOKBACK_DEPTH;
static_assert(kLookbackDepth >= 1 && kLookbackDepth <= 31, "look-back depth must be 1..31");
constexpr uint32_t kTmaPolls = 1u << 22;
// A sequence-parallel fix-up rewrites a tile while the product of a before it
// (from the slice start) exceeds 2^-24 on some channel of the tile: past that
// the carry entering the slice changes no state above fp32 resolution of the
// carry.  The local scan (scan_kernel<..., DEFER>) and the fix-up's preparation both use it.
constexpr float kFixTau = 0x1p-24f;
// Raw input rows a folded SSD conv sees before a warp's first row: up to 4 taps.
constexpr int kConvHalo = 3;
#ifndef NEED_P1_UNROLL
#define NEED_P1_UNROLL 2
#endif
#ifndef NEED_P2_UNROLL
#define NEED_P2_UNROLL 2
#endif
constexpr int kPhase1Unroll = NEED_P1_UNROLL;  // rows per unrolled step of phase 1
constexpr int kPhase2Unroll = NEED_P2_UNROLL;  // and of phase 2
// registers per thread the occupancy bound plans for
// resident CTAs per SM the folded-conv SSD scan is compiled for
#ifndef NEED_CONV_MINB
#define NEED_CONV_MINB 4
#endif
#ifndef NEED_REG_BUDGET
#define NEED_REG_BUDGET 112
#endif

struct ScanParams {
    CUtensorMap tm[5];  // streamed inputs (64-byte aligned members)
    CUtensorMap tm_halo;  // CONV: the raw u rows just before each warp's rows
    int32_t nb, nh, T, C;
    int32_t ncb, nchains, nchunks, ntiles;
    void* out;
    int64_t osb, osh, ost;
    const void* rowdec;  // decay per (b, h, t) when broadcast over C
    int64_t dsb, dsh, dst;
    const float* dskip;
    float dt_min, dt_scale;
    const float* h0;
    float* h_final;
    const uint8_t* seg;
    int64_t sgb, sgt;
    float* summary;
    float* tile_prod;
    float* tile_carry;
    uint32_t* hdr;
    uint32_t lb_polls;  // look-back polls before a wait gives up
    // CONV: the SSD block's causal depthwise conv + SiLU applied to the raw u
    // (in[2]) as it lands: weight [C, K::CONVK] (element strides cwsc, cwsk)
    // and optional bias [C], both in the stream dtype
    const void* conv_w;
    int64_t cwsc, cwsk;
    const void* conv_b;
    // Sequence parallelism.  sp_list / sp_count: the tiles a slice's fix-up
    // rewrites (tile ids as the scan numbers them); the deferring local scan
    // (scan_kernel<K, false, false, true>) appends every tile it defers, the
    // fix-up (scan_kernel<K, true>) reads the first *sp_count entries.
    uint32_t* sp_list;
    uint32_t* sp_count;
    // The fix-up: the local scan's per-tile entering product and state, the
    // gathered slice maps [nranks][nb*nh][C] (prod a, h_end) and this rank.
    const float* fix_tile_prod;
    const float* fix_tile_carry;
    const float2* fix_all_summary;
    int32_t fix_rank;
    ulonglong2* agg;   // [ntiles][8][CBW/8] tagged (A, B): the tile's map
    ulonglong2* incl;  // [ntiles][8][CBW/8] tagged (prod, h): state after the tile
};

// ------------------------------------------------------------------ types
template <typename T>
struct Ops;

template <>
struct Ops<__nv_bfloat16> {
    using P = __nv_bfloat162;
    static constexpr int BYTES = 2;
    static __device__ __forceinline__ P pack(float x, float y) { return __floats2bfloat162_rn(x, y); }
    static __device__ __forceinline__ float2 unpack(P p) { return __bfloat1622float2(p); }
    static __device__ __forceinline__ P mul(P a, P b) { return __hmul2_rn(a, b); }
    static __device__ __forceinline__ P add(P a, P b) { return __hadd2_rn(a, b); }
    static __device__ __forceinline__ P sub(P a, P b) { return __hsub2_rn(a, b); }
    static __device__ __forceinline__ P one() { return __floats2bfloat162_rn(1.0f, 1.0f); }
    static __device__ __forceinline__ P zero() { return __floats2bfloat162_rn(0.0f, 0.0f); }
};

template <>
struct Ops<__half> {
    using P = __half2;
    static constexpr int BYTES = 2;
    static __device__ __forceinline__ P pack(float x, float y) { return __floats2half2_rn(x, y); }
    static __device__ __forceinline__ float2 unpack(P p) { return __half22float2(p); }
    static __device__ __forceinline__ P mul(P a, P b) { return __hmul2_rn(a, b); }
    static __device__ __forceinline__ P add(P a, P b) { return __hadd2_rn(a, b); }
    static __device__ __forceinline__ P sub(P a, P b) { return __hsub2_rn(a, b); }
    static __device__ __forceinline__ P one() { return __floats2half2_rn(1.0f, 1.0f); }
    static __device__ __forceinline__ P zero() { return __floats2half2_rn(0.0f, 0.0f); }
};

template <>
struct Ops<float> {
    using P = float2;
    static constexpr int BYTES = 4;
    static __device__ __forceinline__ P pack(float x, float y) { return make_float2(x, y); }
    static __device__ __forceinline__ float2 unpack(P p) { return p; }
    // separately rounded fp32 ops (no contraction into fma), as torch computes
    static __device__ __forceinline__ P mul(P a, P b) {
        return make_float2(__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y));
    }
    static __device__ __forceinline__ P add(P a, P b) {
        return make_float2(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y));
    }
    static __device__ __forceinline__ P sub(P a, P b) {
        return make_float2(__fsub_rn(a.x, b.x), __fsub_rn(a.y, b.y));
    }
    static __device__ __forceinline__ P one() { return make_float2(1.0f, 1.0f); }
    static __device__ __forceinline__ P zero() { return make_float2(0.0f, 0.0f); }
};

// sigmoid(x) = 1 / (1 + 2^(-x * log2 e)).  16-bit paths round the result to
// bf16/fp16 afterwards, so the hardware ex2/rcp approximations (a few fp32 ulp)
// only move a rounded gate when it lies within those ulp of a rounding tie.
__device__ __forceinline__ float sigmoid_approx(float x) {
    float e, r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(x * -1.4426950408889634f));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.0f + e));
    return r;
}
__device__ __forceinline__ float exp_approx(float x) {
    float e;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(x * 1.4426950408889634f));
    return e;
}
// fp32 paths: library expf and IEEE division, as the reference's fp32 ops.
__device__ __forceinline__ float sigmoid_exact(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x))); }

template <typename T>
__device__ __forceinline__ float sigm(float x) {
    if constexpr (Ops<T>::BYTES == 4) return sigmoid_exact(x);
    else return sigmoid_approx(x);
}
template <typename T>
__device__ __forceinline__ float expo(float x) {
    if constexpr (Ops<T>::BYTES == 4) return expf(x);
    else return exp_approx(x);
}

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }

// ------------------------------------------------------------------ packed fp32 pairs
// sm_100 executes these as single f32x2 instructions (FFMA2 / FMUL2 / FADD2);
// each lane is an ordinary IEEE round-to-nearest fp32 op.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 splat2(float v) { return make_float2(v, v); }

// a packed 16-bit pair (or an fp32 pair) as two fp32 values
__device__ __forceinline__ float2 widen(__nv_bfloat162 p) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(&p);
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
__device__ __forceinline__ float2 widen(__half2 p) { return __half22float2(p); }
__device__ __forceinline__ float2 widen(float2 p) { return p; }

// sigmoid / exp of a pair: 16-bit paths use the hardware approximations (the
// result is rounded to 16 bits next), fp32 paths the library exp and IEEE division
template <typename T>
__device__ __forceinline__ float2 sig2(float2 x) {
    if constexpr (Ops<T>::BYTES == 4) {
        return make_float2(sigmoid_exact(x.x), sigmoid_exact(x.y));
    } else {
        const float2 t = fmul2(x, splat2(-1.4426950408889634f));
        float e0, e1, r0, r1;
        asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(t.x));
        asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(t.y));
        const float2 d = fadd2(make_float2(e0, e1), splat2(1.0f));
        asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r0) : "f"(d.x));
        asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r1) : "f"(d.y));
        return make_float2(r0, r1);
    }
}
template <typename T>
__device__ __forceinline__ float2 exp2_pair(float2 x) {  // exp(x) of a pair
    if constexpr (Ops<T>::BYTES == 4) {
        return make_float2(expf(x.x), expf(x.y));
    } else {
        const float2 t = fmul2(x, splat2(1.4426950408889634f));
        float e0, e1;
        asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(t.x));
        asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(t.y));
        return make_float2(e0, e1);
    }
}

// ------------------------------------------------------------------ 8-channel rows
// A thread's 8 channels: with SPLIT (any 4-byte stream) they are two groups of
// four, channels [lane*4, +4) and [128 + lane*4, +4); otherwise one group of
// eight, [lane*8, +8).  Pair i holds channels (2i, 2i+1) of that list.
template <bool SPLIT>
__device__ __forceinline__ int chan(int e, int lane) {
    return SPLIT ? ((e >> 2) * 128 + lane * 4 + (e & 3)) : (lane * 8 + e);
}

template <typename T, bool SPLIT>
struct Row8 {
    using P = typename Ops<T>::P;
    // shared -> 4 pairs
    static __device__ __forceinline__ void lds(const T* row, int lane, P (&p)[4]) {
        if constexpr (Ops<T>::BYTES == 4) {
            const float4 v0 = *reinterpret_cast<const float4*>(row + lane * 4);
            const float4 v1 = *reinterpret_cast<const float4*>(row + 128 + lane * 4);
            p[0] = make_float2(v0.x, v0.y);
            p[1] = make_float2(v0.z, v0.w);
            p[2] = make_float2(v1.x, v1.y);
            p[3] = make_float2(v1.z, v1.w);
        } else if constexpr (SPLIT) {
            const uint2 v0 = *reinterpret_cast<const uint2*>(row + lane * 4);
            const uint2 v1 = *reinterpret_cast<const uint2*>(row + 128 + lane * 4);
            const uint32_t w[4] = {v0.x, v0.y, v1.x, v1.y};
#pragma unroll
            for (int i = 0; i < 4; ++i) p[i] = *reinterpret_cast<const P*>(&w[i]);
        } else {
            const uint4 v = *reinterpret_cast<const uint4*>(row + lane * 8);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) p[i] = *reinterpret_cast<const P*>(&w[i]);
        }
    }
    static __device__ __forceinline__ void sts(T* row, int lane, const P (&p)[4]) {
        if constexpr (Ops<T>::BYTES == 4) {
            *reinterpret_cast<float4*>(row + lane * 4) = make_float4(p[0].x, p[0].y, p[1].x, p[1].y);
            *reinterpret_cast<float4*>(row + 128 + lane * 4) = make_float4(p[2].x, p[2].y, p[3].x, p[3].y);
        } else {
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) w[i] = *reinterpret_cast<const uint32_t*>(&p[i]);
            if constexpr (SPLIT) {
                *reinterpret_cast<uint2*>(row + lane * 4) = make_uint2(w[0], w[1]);
                *reinterpret_cast<uint2*>(row + 128 + lane * 4) = make_uint2(w[2], w[3]);
            } else {
                *reinterpret_cast<uint4*>(row + lane * 8) = make_uint4(w[0], w[1], w[2], w[3]);
            }
        }
    }
    // registers -> global row (channel 0 of the tile at `row`); group g is
    // stored only when ok[g] (channels past C are never written)
    static __device__ __forceinline__ void stg(T* row, int lane, const P (&p)[4], bool ok0, bool ok1) {
        if constexpr (Ops<T>::BYTES == 4) {
            if (ok0) *reinterpret_cast<float4*>(row + lane * 4) = make_float4(p[0].x, p[0].y, p[1].x, p[1].y);
            if (ok1) *reinterpret_cast<float4*>(row + 128 + lane * 4) = make_float4(p[2].x, p[2].y, p[3].x, p[3].y);
        } else {
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) w[i] = *reinterpret_cast<const uint32_t*>(&p[i]);
            if constexpr (SPLIT) {
                if (ok0) *reinterpret_cast<uint2*>(row + lane * 4) = make_uint2(w[0], w[1]);
                if (ok1) *reinterpret_cast<uint2*>(row + 128 + lane * 4) = make_uint2(w[2], w[3]);
            } else {
                if (ok0) *reinterpret_cast<uint4*>(row + lane * 8) = make_uint4(w[0], w[1], w[2], w[3]);
            }
        }
    }
};

// ------------------------------------------------------------------ config
// FORM, stream dtype TS, decay dtype TD (AFFINE / RETENTION), decay broadcast
// over channels (ROWDEC), tokens per tile L, row warps NW, channels per tile CBW.
// A lane owns 8 channels; a row of a tile takes LPR = CBW/8 lanes, so a warp
// works on SS = 32/LPR rows side by side.
template <int FORM_, typename TS_, typename TD_, bool ROWDEC_, int L_, int NW_, int CBW_ = 256, int CONVK_ = 0>
struct ScanCfg {
    static constexpr int FORM = FORM_;
    using TS = TS_;  // streamed dtype (inputs other than a separate decay, and the output)
    using TD = TD_;  // decay dtype (AFFINE / RETENTION)
    static constexpr bool ROWDEC = ROWDEC_;
    static constexpr int L = L_, NW = NW_, CBW = CBW_, R = L / NW;
    static constexpr int LB = NW;  // the look-back warp (after the NW row warps)
    static constexpr int NT = (NW + 1) * 32;
    static constexpr bool HAS_DSTREAM = (FORM == FORM_AFFINE || FORM == FORM_RETENTION) && !ROWDEC;
    static constexpr bool SPLIT = (Ops<TS>::BYTES == 4) || (HAS_DSTREAM && Ops<TD>::BYTES == 4);
    static constexpr int LPR = CBW / 8, SS = 32 / LPR, RS = R / SS;  // lanes per row, rows side by side, rows per thread
    static_assert(L % NW == 0 && R % SS == 0, "rows must split evenly over warps and lanes");
    static_assert(!SPLIT || CBW == 256, "4-byte streams use 256-channel tiles");
    static_assert(CBW == 64 || CBW == 128 || CBW == 256, "64, 128 or 256 channels per tile");
    static_assert(R <= 32, "a warp loads the reset flags of its rows one per lane");
    // streamed inputs, in[] order of the C ABI
    static constexpr int NIN = FORM == FORM_AFFINE      ? (ROWDEC ? 1 : 2)
                               : FORM == FORM_GATED     ? 3
                               : FORM == FORM_SSD       ? 5
                                                        : (ROWDEC ? 2 : 3);
    // in[] index of the first streamed tensor (AFFINE/RETENTION with a row decay skip in[0])
    static constexpr int IN0 = ((FORM == FORM_AFFINE || FORM == FORM_RETENTION) && ROWDEC) ? 1 : 0;
    __host__ __device__ static constexpr int slot_bytes(int k) {
        return L * CBW * ((HAS_DSTREAM && k == 0) ? Ops<TD>::BYTES : Ops<TS>::BYTES);
    }
    __host__ __device__ static constexpr int slots_bytes() {
        int s = 0;
        for (int k = 0; k < NIN; ++k) s += slot_bytes(k);
        return s;
    }
    // GATED frees its input-gate slot after phase 1: the warp maps live there.
    static constexpr int AGG_SLOT = FORM == FORM_GATED ? 1 : -1;
    static constexpr int AGG_BYTES = NW * 4 * 32 * 16;  // per warp: 4 pairs x 32 lanes x (A2, B2)
    // warp maps: in the freed slot each warp's map sits in that warp's own rows
    // (no barrier needed before writing it); otherwise packed
    static constexpr int AGG_STRIDE = AGG_SLOT >= 0 ? (L * CBW * Ops<TS>::BYTES / NW) : 4 * 32 * 16;
    static_assert(AGG_SLOT < 0 || AGG_STRIDE >= 4 * 32 * 16, "a warp's rows must hold its map");
    static constexpr int OFF_AGG = slots_bytes();
    static constexpr int OFF_HIN = OFF_AGG + (AGG_SLOT < 0 ? AGG_BYTES : 0);
    static constexpr int OFF_ROWDEC = OFF_HIN + NW * CBW * 4;  // fp32 state entering each warp's rows
    static constexpr int OFF_RESET = OFF_ROWDEC + (ROWDEC ? L * 4 : 0);
    // CONV (16-bit SSD): per warp the kConvHalo raw u rows before its rows (a
    // TMA box, 128-byte aligned) and the reset flags of rows wr0-kConvHalo ..
    // wr0+R-1 (32 bytes)
    static constexpr int CONVK = CONVK_;  // taps of the folded conv (0: none)
    static constexpr bool CONV = CONVK > 0;
    static_assert(CONVK >= 0 && CONVK <= kConvHalo + 1, "1 .. kConvHalo + 1 taps");
    static_assert(!CONV || (FORM == FORM_SSD && Ops<TS>::BYTES == 2), "the conv fold is for 16-bit SSD");
    static_assert(!CONV || R + kConvHalo <= 32, "a warp loads its conv reset flags one per lane");
    static_assert(!CONV || kConvHalo <= RS, "a thread's window rows lie in its own or the previous row group");
    static constexpr int OFF_HALO =
        CONV ? (((OFF_RESET + ((L + 15) / 16) * 16) + 127) / 128) * 128 : OFF_RESET + ((L + 15) / 16) * 16;
    static constexpr int HALO_WARP_BYTES = kConvHalo * CBW * Ops<TS>::BYTES;
    static constexpr int OFF_CRESET = OFF_HALO + (CONV ? NW * HALO_WARP_BYTES : 0);
    static constexpr int OFF_MISC = OFF_CRESET + (CONV ? NW * 32 : 0);
    static constexpr int SMEM = OFF_MISC + (NW + 1) * 8 + 16 + 128;  // mbarriers, misc, alignment slack
    // resident CTAs per SM: bounded by shared memory (228 KB per SM, 1 KB
    // reserved per CTA) and by a register budget per thread
    static constexpr int MINB_SMEM = (228 * 1024) / (SMEM + 1024);
    static constexpr int MINB_REGS = 65536 / (NT * NEED_REG_BUDGET);
    static constexpr int MINB_CAP = MINB_REGS < 1 ? 1 : (MINB_REGS > 8 ? 8 : MINB_REGS);
    static constexpr int MINB_PLAIN = MINB_SMEM < 1 ? 1 : (MINB_SMEM < MINB_CAP ? MINB_SMEM : MINB_CAP);
    static constexpr int MINB = CONV ? (NEED_CONV_MINB < MINB_SMEM ? NEED_CONV_MINB : MINB_SMEM) : MINB_PLAIN;
};

template <class K>
__device__ __forceinline__ unsigned char* slot_ptr(unsigned char* base, int k) {
    int off = 0;
#pragma unroll
    for (int j = 0; j < 5; ++j)
        if (j < k) off += K::slot_bytes(j);
    return base + off;
}

// ------------------------------------------------------------------ folded conv
// CONV: as the rows land, the raw u in the tile's u slot (slot 2) becomes
// u = SiLU(round(conv(raw))) rounded to the stream dtype, the arithmetic of
// prologue.cu's conv_silu_kernel bit for bit: the taps accumulated oldest
// first by fp32 fma onto the bias, rounded, SiLU with the scan's 16-bit
// sigmoid, rounded.  Rows before the sequence start read as 0 (the halo box's
// zero fill); a reset at row t (a segment start) hides every row before t from
// the taps of rows >= t.  A pass between the rows' arrival and phase 1 does
// it (merged into phase 1's row loop it measured slower: 72.5 against 67.7 us
// at B=8, T=2048, C=832); the rows before a thread's first row come from the
// previous row group of its warp or, for the first, from the warp's halo.
// This lane's tap weights by distance back from the current row (0 past
// K::CONVK) and biases, as fp32 pairs; loaded before the tile lands.
struct ConvTaps {
    float2 wb[kConvHalo + 1][4], bs[4];
};
template <class K>
__device__ __forceinline__ void conv_taps(const ScanParams& p, int v, int c0, ConvTaps& ct) {
    using TS = typename K::TS;
    constexpr int kc = K::CONVK;
    const TS* w = static_cast<const TS*>(p.conv_w);
    const TS* bias = static_cast<const TS*>(p.conv_b);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int ca = c0 + chan<false>(2 * i, v), cb = ca + 1;
        const bool oa = ca < p.C, ob = cb < p.C;
        ct.bs[i] = make_float2(bias != nullptr && oa ? to_f(bias[ca]) : 0.0f,
                               bias != nullptr && ob ? to_f(bias[cb]) : 0.0f);
#pragma unroll
        for (int back = 0; back <= kConvHalo; ++back) {
            const int64_t j = kc - 1 - back;  // tap index (oldest first)
            ct.wb[back][i] = make_float2(back < kc && oa ? to_f(w[ca * p.cwsc + j * p.cwsk]) : 0.0f,
                                         back < kc && ob ? to_f(w[cb * p.cwsc + j * p.cwsk]) : 0.0f);
        }
    }
}

// One output row of the folded conv for this lane's 8 channels: jr is the
// row's index in the thread's window numbering (its rows are kConvHalo ..
// kConvHalo+RS-1), win[] the raw rows jr-3 .. jr-1 (oldest first), raw the
// row itself; taps from rows before `lastres` are outside the row's segment.
template <class K>
__device__ __forceinline__ void conv_row(const ConvTaps& ct, int jr, int lastres,
                                         const typename Ops<typename K::TS>::P (&win)[kConvHalo][4],
                                         const typename Ops<typename K::TS>::P (&raw)[4],
                                         typename Ops<typename K::TS>::P (&o)[4]) {
    using TS = typename K::TS;
    using OS = Ops<TS>;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 acc = ct.bs[i];
#pragma unroll
        for (int back = K::CONVK - 1; back >= 0; --back) {
            {
                const float2 x = jr - back >= lastres ? widen(back == 0 ? raw[i] : win[kConvHalo - back][i])
                                                      : splat2(0.0f);
                acc = ffma2(ct.wb[back][i], x, acc);
            }
        }
        const float2 a = widen(OS::pack(acc.x, acc.y));
        const float2 y = fmul2(a, sig2<TS>(a));
        o[i] = OS::pack(y.x, y.y);
    }
}

// The folded conv over this thread's rows r0 .. r0+RS-1 of the u slot, in
// place: all window rows are read first (one warp barrier), then each row is
// rewritten.
template <class K>
__device__ __forceinline__ void conv_fold(const ScanParams& p, unsigned char* base, int warp, int q, int v, int wr0,
                                          const ConvTaps& ct) {
    using TS = typename K::TS;
    using PS = typename Ops<TS>::P;
    constexpr int RS = K::RS, CBW = K::CBW, H = kConvHalo;
    const int r0 = wr0 + q * RS;
    TS* slot = reinterpret_cast<TS*>(slot_ptr<K>(base, 2));
    const TS* halo = reinterpret_cast<const TS*>(base + K::OFF_HALO + warp * K::HALO_WARP_BYTES);
    const uint8_t* rsf = base + K::OFF_CRESET + warp * 32 + q * RS;  // flag of window row jr: rsf[jr]
    PS raw[RS + H][4];  // window row jr = row r0 - H + jr
#pragma unroll
    for (int jr = 0; jr < RS + H; ++jr) {
        const int r = r0 - H + jr;
        Row8<TS, false>::lds(r >= wr0 ? slot + r * CBW : halo + (r - wr0 + H) * CBW, v, raw[jr]);
    }
    __syncwarp();
    int lastres = 0;  // taps from window rows >= lastres are inside the current row's segment
#pragma unroll
    for (int jr = 1; jr < H; ++jr)
        if (rsf[jr]) lastres = jr;
#pragma unroll
    for (int jo = 0; jo < RS; ++jo) {
        const int jr = H + jo;
        if (rsf[jr]) lastres = jr;
        PS win[H][4], o[4];
#pragma unroll
        for (int jw = 0; jw < H; ++jw)
#pragma unroll
            for (int i = 0; i < 4; ++i) win[jw][i] = raw[jo + jw][i];
        conv_row<K>(ct, jr, lastres, win, raw[jr], o);
        Row8<TS, false>::sts(slot + (r0 + jo) * CBW, v, o);
    }
    __syncwarp();
}

// ------------------------------------------------------------------ the kernel
// FIX = false: the scan, one tile per CTA.  FIX = true: the sequence-parallel
// fix-up -- the same tile pipeline over the fix_count tiles of fix_list (the
// leading tiles of each chain of a slice), each tile entered from its known
// corrected state (no look-back), the resident CTAs striding over the list.
// REV = true (AFFINE only, no resets): the scan runs from t = T-1 down to 0,
// h_t = a'_t h_{t+1} + b_t -- the adjoint recurrence of the backward pass.
// Tiles, rows and the look-back work in reversed ("virtual") time tau =
// T-1-t; only the tile loads, the row order inside a warp's rows and the
// output rows are mirrored.  The caller passes the decay already shifted by
// one row (a'_t = a_{t+1}, a'_{T-1} = 0): a tensor map based at row 1 with
// T-1 rows, or, for a decay per row, a guarded load of row t+1.
// DEFER = true: the local scan of a sequence-parallel slice after the first --
// tiles whose entering product of a exceeds kFixTau on some channel skip
// phase 2 (the fix-up writes their outputs; it rewrites exactly those tiles).
template <class K, bool FIX = false, bool REV = false, bool DEFER = false>
__global__ void __launch_bounds__(K::NT, K::MINB) scan_kernel(const __grid_constant__ ScanParams p) {
    using TS = typename K::TS;
    using TD = typename K::TD;
    using OS = Ops<TS>;
    using PS = typename OS::P;
    constexpr bool SPLIT = K::SPLIT;
    constexpr int L = K::L, NW = K::NW, R = K::R, CBW = K::CBW, LPR = K::LPR, SS = K::SS, RS = K::RS;

    extern __shared__ unsigned char smem_raw[];
    unsigned char* base = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    unsigned char* s_agg = K::AGG_SLOT >= 0 ? slot_ptr<K>(base, K::AGG_SLOT) : base + K::OFF_AGG;
    float* s_hin = reinterpret_cast<float*>(base + K::OFF_HIN);  // [NW][CBW] state entering each warp
    float* s_rowdec = reinterpret_cast<float*>(base + K::OFF_ROWDEC);
    uint8_t* s_reset = base + K::OFF_RESET;
    uint64_t* s_bar = reinterpret_cast<uint64_t*>(base + K::OFF_MISC);  // one per row warp
    uint64_t* s_p1 = s_bar + NW;  // all row warps have written their maps
    uint32_t* s_defer = reinterpret_cast<uint32_t*>(s_p1 + 1);  // DEFER: this tile skips phase 2
    // warp w's maps: 4 pairs x 32 lanes of (A pair, B pair); lane = (row group, channel vector)
    auto agg4 = [&](int w) { return reinterpret_cast<float4*>(s_agg + w * K::AGG_STRIDE); };

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int v = lane % LPR;  // channel vector (8 channels) of this lane
    const int q = lane / LPR;  // row group of this lane within its warp

    // Tile ids follow blockIdx.x (chunk-major).  CTAs are dispatched in
    // increasing blockIdx order, so every tile a CTA waits on belongs to a CTA
    // that is already resident or finished -- the property single-pass
    // decoupled look-back scans rely on; the waits are bounded regardless.
    if (tid == 0) {
        for (int w = 0; w < NW; ++w) mbar_init(&s_bar[w], 1);
        mbar_init(s_p1, NW * 32);
        fence_barrier_init();
    }
    __syncthreads();
    const int ntl = FIX ? min(p.ntiles, static_cast<int>(*p.sp_count)) : p.ntiles;
    const int stride = FIX ? static_cast<int>(gridDim.x) : p.ntiles;
    uint32_t par = 0;  // mbarrier phase of this CTA's current tile
    // FIX: entry `item` of the list names the tile; the next entry is read one tile ahead
    int next_tile = static_cast<int>(blockIdx.x);
    if (FIX && next_tile < ntl) next_tile = static_cast<int>(p.sp_list[next_tile]);
    for (int item = static_cast<int>(blockIdx.x); item < ntl; item += stride, par ^= 1u) {
        const int tile = next_tile;
        if (FIX && item + stride < ntl) next_tile = static_cast<int>(p.sp_list[item + stride]);
        if (FIX && static_cast<unsigned>(tile) >= static_cast<unsigned>(p.ntiles)) {
            // not a tile of this slice (a list no deferring local scan wrote):
            // report it and skip, leaving the barriers' phase where it was
            if (threadIdx.x == 0) atomicOr(&p.hdr[WS_ERROR], ERR_SP_LIST);
            par ^= 1u;
            continue;
        }
        const int chunk = tile / p.nchains;
        const int chain = tile - chunk * p.nchains;
        const int seq = chain / p.ncb;
        const int cblk = chain - seq * p.ncb;
        const int bi = seq / p.nh, hi = seq - bi * p.nh;
        const int t0 = chunk * L, c0 = cblk * CBW;
        const int nvalid = min(L, p.T - t0);  // rows of this tile inside T

        // The look-back warp's layout: each lane owns NE = 8 / SS channels of one
        // channel vector -- elements q*NE .. q*NE+NE-1 of vector v -- so all 32
        // lanes work; NP = NE / 2 channel pairs.
        constexpr int NE = 8 / SS, NP = NE / 2;
        auto lbchan = [&](int k) { return chan<SPLIT>(q * NE + k, v); };  // channel of element k
        // warp w's total map (the in-warp inclusive map of its last row group)
        // for this lane's pair k
        auto wtotal = [&](int w, int k) { return agg4(w)[(q * NP + k) * 32 + (SS - 1) * LPR + v]; };
        // One pass over the warp totals in row order, each batch of WB warps'
        // loads issued ahead of the chain: with `hand`, walks h (the carry entering the tile)
        // through them, leaving in s_hin the state entering each warp's rows, and
        // releases the row warps; with `comp`, composes this tile's map (TA, TB).
        constexpr int WB = NP >= 4 ? 2 : 4;  // warps per batch of map loads (8 float4 in flight)
        auto pass = [&](float (&h)[NE], float2 (&TA)[NP], float2 (&TB)[NP], bool hand, bool comp) {
            if (comp) {
#pragma unroll
                for (int k = 0; k < NP; ++k) {
                    TA[k] = splat2(1.0f);
                    TB[k] = splat2(0.0f);
                }
            }
#pragma unroll
            for (int w0 = 0; w0 < NW; w0 += WB) {
                float4 m[WB][NP];
#pragma unroll
                for (int dw = 0; dw < WB; ++dw)
#pragma unroll
                    for (int k = 0; k < NP; ++k)
                        if (w0 + dw < NW) m[dw][k] = wtotal(w0 + dw, k);
#pragma unroll
                for (int dw = 0; dw < WB; ++dw) {
                    if (w0 + dw >= NW) break;
                    if (hand) {
                        float* dst = s_hin + (w0 + dw) * CBW;
                        if constexpr (NE >= 4) {
#pragma unroll
                            for (int g = 0; g < NE / 4; ++g)
                                *reinterpret_cast<float4*>(dst + lbchan(4 * g)) =
                                    make_float4(h[4 * g], h[4 * g + 1], h[4 * g + 2], h[4 * g + 3]);
                        } else {
                            *reinterpret_cast<float2*>(dst + lbchan(0)) = make_float2(h[0], h[1]);
                        }
                    }
#pragma unroll
                    for (int k = 0; k < NP; ++k) {
                        const float4 mm = m[dw][k];
                        if (hand) {
                            h[2 * k] = fmaf(mm.x, h[2 * k], mm.z);
                            h[2 * k + 1] = fmaf(mm.y, h[2 * k + 1], mm.w);
                        }
                        if (comp) {
                            TB[k] = ffma2(make_float2(mm.x, mm.y), TB[k], make_float2(mm.z, mm.w));
                            TA[k] = fmul2(make_float2(mm.x, mm.y), TA[k]);
                        }
                    }
                }
            }
            if (hand) {
                __syncwarp();
                named_arrive(1, K::NT);  // the row warps may run phase 2
            }
        };
        auto el = [](const float2 (&x)[NP], int k) { return (k & 1) ? x[k >> 1].y : x[k >> 1].x; };

        if (FIX && warp == K::LB) {
            // ------------------------------------------------------ fix-up carry
            // The carry entering the slice, composed from the gathered maps of the
            // ranks before this one (8 maps in flight at a time, identity maps past
            // the last); the state entering this tile of the slice is the local
            // scan's state plus that carry times the product of a before the tile.
            // The chain's first tile also writes the slice's corrected final state
            // and summary.
            const int64_t nsc = (int64_t)p.nb * p.nh * p.C;
            float carry[NE];
#pragma unroll
            for (int k = 0; k < NE; ++k) carry[k] = 0.0f;
            for (int j0 = 0; j0 < p.fix_rank; j0 += 8) {
#pragma unroll
                for (int k = 0; k < NE; ++k) {
                    const int c = c0 + lbchan(k);
                    float2 m[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        m[j] = (j0 + j < p.fix_rank && c < p.C)
                                   ? p.fix_all_summary[(j0 + j) * nsc + (int64_t)seq * p.C + c]
                                   : make_float2(1.0f, 0.0f);
#pragma unroll
                    for (int j = 0; j < 8; ++j) carry[k] = fmaf(m[j].x, carry[k], m[j].y);
                }
            }
            const int64_t ti0 = ((int64_t)seq * p.nchunks + chunk) * p.C;
            float h[NE];
#pragma unroll
            for (int k = 0; k < NE; ++k) {
                const int c = c0 + lbchan(k);
                h[k] = c < p.C ? fmaf(p.fix_tile_prod[ti0 + c], carry[k], p.fix_tile_carry[ti0 + c]) : 0.0f;
                if (chunk == 0 && c < p.C) {
                    const float2 mine = p.fix_all_summary[p.fix_rank * nsc + (int64_t)seq * p.C + c];
                    const float hl = fmaf(mine.x, carry[k], mine.y);
                    if (p.h_final != nullptr) p.h_final[(int64_t)seq * p.C + c] = hl;
                    if (p.summary != nullptr)
                        reinterpret_cast<float2*>(p.summary)[(int64_t)seq * p.C + c] = make_float2(mine.x, hl);
                }
            }
            if (!mbar_wait_bounded(s_p1, par, kTmaPolls)) atomicOr(&p.hdr[WS_ERROR], ERR_TMA);
            float2 TA[NP], TB[NP];
            pass(h, TA, TB, true, false);
        } else if (warp == K::LB) {
            // ------------------------------------------------------ look-back warp
            // It owns no rows.  From the start of the CTA it polls the predecessors'
            // records -- the maps of the up to kLookbackDepth tiles before this one
            // and the inclusive state of the tile before those, composed in that
            // fixed order, so results are bit-reproducible -- while the row warps
            // load and run phase 1.  When the warps' totals are in it composes this
            // tile's map and publishes it (AGG) -- never held back by a predecessor
            // -- and, with the carry known (usually by then), in the same pass hands
            // the row warps their entering states (named barrier); then it publishes
            // the inclusive state.  Records carry the launch epoch in every 64-bit
            // word, so publishing needs no fence and a poll returns the data itself.
            uint32_t ep = 0;
            if (lane == 0) {
                // Every CTA of a launch gets the same epoch: the low half counts CTAs
                // in, and the last one to start moves the epoch on for the next launch.
                unsigned long long* lw = reinterpret_cast<unsigned long long*>(p.hdr + WS_LAUNCH);
                const unsigned long long old = atomicAdd(lw, 1ull);
                if (static_cast<uint32_t>(old) == static_cast<uint32_t>(p.ntiles) - 1u)
                    atomicAdd(lw, (1ull << 32) - static_cast<unsigned long long>(p.ntiles));
                ep = static_cast<uint32_t>(old >> 32);
            }
            const uint32_t tag = (__shfl_sync(0xffffffffu, ep, 0) & 0x7fffffffu) | 0x80000000u;
            float carry[NE], carryP[NE];
            float2 TA[NP], TB[NP];  // this tile's map
            const int nagg = chunk == 0 ? 0 : min(chunk - 1, kLookbackDepth);
            bool pread = chunk == 0, mapped = false, agg_pub = chunk == 0;  // chunk 0 publishes no bare map
            bool handed = false;
            if (chunk == 0) {
#pragma unroll
                for (int k = 0; k < NE; ++k) {
                    const int c = c0 + lbchan(k);
                    carry[k] = (p.h0 != nullptr && c < p.C) ? p.h0[(int64_t)seq * p.C + c] : 0.0f;
                    carryP[k] = 1.0f;
                }
            }
            ulonglong2* const my_agg = p.agg + (int64_t)tile * CBW;
            // DEFER: with the product before this tile known, does some channel
            // still exceed kFixTau (then the fix-up writes the outputs)?  Written to
            // s_defer before the row warps are released.
            auto set_defer = [&]() {
                if constexpr (DEFER) {
                    bool d = false;
#pragma unroll
                    for (int k = 0; k < NE; ++k) d |= (c0 + lbchan(k) < p.C) && carryP[k] > kFixTau;
                    d = __any_sync(0xffffffffu, d);
                    if (lane == 0) {
                        *s_defer = d ? 1u : 0u;
                        if (d) p.sp_list[atomicAdd(p.sp_count, 1u)] = static_cast<uint32_t>(tile);  // for the fix-up
                    }
                }
            };
            auto publish_agg = [&]() {
#pragma unroll
                for (int k = 0; k < NE; ++k)
                    st_relaxed_v2u64(&my_agg[(q * NE + k) * LPR + v], tagged(el(TA, k), tag), tagged(el(TB, k), tag));
                agg_pub = true;
            };
            bool ok = false;
            for (uint32_t it = 0; it < p.lb_polls; ++it) {
                bool progressed = false;
                if (!pread) {
                    bool valid = true;
                    float accA[NE], accB[NE];
#pragma unroll
                    for (int k = 0; k < NE; ++k) {
                        accA[k] = 1.0f;
                        accB[k] = 0.0f;
                    }
                    for (int j = 0; j < nagg; ++j) {
                        const ulonglong2* src = p.agg + (int64_t)(tile - (j + 1) * p.nchains) * CBW;
#pragma unroll
                        for (int k = 0; k < NE; ++k) {
                            const ulonglong2 m = ld_relaxed_v2u64(&src[(q * NE + k) * LPR + v]);  // (A, B)
                            valid &= tag_ok(m.x, tag) & tag_ok(m.y, tag);
                            accB[k] = fmaf(accA[k], untag(m.y), accB[k]);
                            accA[k] = accA[k] * untag(m.x);
                        }
                    }
                    const ulonglong2* src = p.incl + (int64_t)(tile - (nagg + 1) * p.nchains) * CBW;
#pragma unroll
                    for (int k = 0; k < NE; ++k) {
                        const ulonglong2 m = ld_relaxed_v2u64(&src[(q * NE + k) * LPR + v]);  // (prod, h)
                        valid &= tag_ok(m.x, tag) & tag_ok(m.y, tag);
                        carry[k] = fmaf(accA[k], untag(m.y), accB[k]);
                        carryP[k] = accA[k] * untag(m.x);
                    }
                    if (__all_sync(0xffffffffu, valid)) pread = progressed = true;
                }
                // with the carry in, nothing else is polled: suspend on the barrier
                // (try_wait wakes when the phase completes) instead of spinning
                if (!mapped && __all_sync(0xffffffffu, pread ? mbar_try_wait(s_p1, par) : mbar_test_wait(s_p1, par))) {
                    float h[NE];
#pragma unroll
                    for (int k = 0; k < NE; ++k) h[k] = carry[k];
                    if (pread) set_defer();
                    pass(h, TA, TB, pread, true);  // with the carry in, the hand-out rides along
                    handed = pread;
                    mapped = progressed = true;
                    if (!agg_pub) publish_agg();  // successors may compose this map before our carry is in
                }
                if (mapped && pread) {
                    ok = true;
                    break;
                }
                if (!progressed && !pread && it >= 2) __nanosleep(64);
                if ((it & 1023u) == 1023u && ld_volatile_u32(&p.hdr[WS_ERROR]) != 0) break;  // fail fast
            }
            if (!ok) {
                if (lane == 0) atomicOr(&p.hdr[WS_ERROR], ERR_LOOKBACK);
                if (!pread) {
#pragma unroll
                    for (int k = 0; k < NE; ++k) {
                        carry[k] = 0.0f;
                        carryP[k] = 0.0f;
                    }
                }
                if (!mapped) {
                    mbar_wait_bounded(s_p1, par, kTmaPolls);
                    float h[NE];
                    pass(h, TA, TB, false, true);
                }
            }
            if (!handed) {
                float h[NE];
#pragma unroll
                for (int k = 0; k < NE; ++k) h[k] = carry[k];
                set_defer();
                pass(h, TA, TB, true, false);
            }
            // the inclusive state: for the successors kLookbackDepth + 1 chunks on,
            // the final state, the slice summary and the per-tile products
            float inclP[NE], inclH[NE];
#pragma unroll
            for (int k = 0; k < NE; ++k) {
                inclP[k] = el(TA, k) * carryP[k];
                inclH[k] = fmaf(el(TA, k), carry[k], el(TB, k));
            }
            if (chunk + 1 < p.nchunks) {
                if (!agg_pub) publish_agg();
                ulonglong2* mi = p.incl + (int64_t)tile * CBW;
#pragma unroll
                for (int k = 0; k < NE; ++k)
                    st_relaxed_v2u64(&mi[(q * NE + k) * LPR + v], tagged(inclP[k], tag), tagged(inclH[k], tag));
            }
#pragma unroll
            for (int k = 0; k < NE; ++k) {
                const int c = c0 + lbchan(k);
                if (c < p.C) {
                    const int64_t ti = ((int64_t)seq * p.nchunks + chunk) * p.C + c;
                    if (p.tile_prod != nullptr) p.tile_prod[ti] = carryP[k];
                    if (p.tile_carry != nullptr) p.tile_carry[ti] = carry[k];
                    if (chunk + 1 == p.nchunks) {
                        if (p.h_final != nullptr) p.h_final[(int64_t)seq * p.C + c] = inclH[k];
                        if (p.summary != nullptr)
                            reinterpret_cast<float2*>(p.summary)[(int64_t)seq * p.C + c] =
                                make_float2(inclP[k], inclH[k]);
                    }
                }
            }
        } else {
        // ---------------------------------------------------------- row warps
        // Each warp loads its own R rows (one TMA box per input) and starts on them
        // as soon as they land, so compute overlaps the rest of the tile's load.
        const int wr0 = warp * R;                              // this warp's first row
        const int r0 = wr0 + q * RS;                           // this thread's first row
        const int rend = max(0, min(RS, nvalid - r0));         // this thread's rows inside T
        if (lane == 0 && nvalid > wr0 && FIX && K::FORM == FORM_GATED) {
            // the gated fix-up: z, and the rounded b the deferring local scan left in
            // the tile's output rows (p.tm[3]); the input gate's slot is not loaded
            mbar_arrive_expect_tx(&s_bar[warp], (K::slot_bytes(0) + K::slot_bytes(2)) / NW);
            tma_load_4d(slot_ptr<K>(base, 0) + wr0 * (K::slot_bytes(0) / L), &p.tm[0], c0, t0 + wr0, hi, bi,
                        &s_bar[warp]);
            tma_load_4d(slot_ptr<K>(base, 2) + wr0 * (K::slot_bytes(2) / L), &p.tm[3], c0, t0 + wr0, hi, bi,
                        &s_bar[warp]);
        } else if (lane == 0 && nvalid > wr0) {
            uint32_t bytes = 0;
#pragma unroll
            for (int k = 0; k < K::NIN; ++k) bytes += K::slot_bytes(k) / NW;
            if constexpr (K::CONV) bytes += K::HALO_WARP_BYTES;
            mbar_arrive_expect_tx(&s_bar[warp], bytes);
#pragma unroll
            for (int k = 0; k < K::NIN; ++k)
                tma_load_4d(slot_ptr<K>(base, k) + wr0 * (K::slot_bytes(k) / L), &p.tm[k], c0,
                            REV ? p.T - t0 - wr0 - R : t0 + wr0, hi, bi,
                            &s_bar[warp]);
            // the raw u rows before this warp's rows (a negative row reads the zero fill)
            if constexpr (K::CONV)
                tma_load_4d(base + K::OFF_HALO + warp * K::HALO_WARP_BYTES, &p.tm_halo, c0, t0 + wr0 - kConvHalo,
                            hi, bi, &s_bar[warp]);
        }
        // this warp's reset flags and per-row decay while its rows are in flight
        if (lane < R) {
            const int r = wr0 + lane, t = t0 + r;
            uint8_t rs = 0;
            if (!REV && p.seg != nullptr && t < p.T) rs = p.seg[bi * p.sgb + (int64_t)t * p.sgt] != 0;
            s_reset[r] = rs;
            if constexpr (K::ROWDEC) {
                float d = 1.0f;
                if (t < p.T) {
                    // REV: the decay of the row after this one in time (0 past the end)
                    const int tt = REV ? p.T - t : t;
                    d = tt < p.T ? to_f(reinterpret_cast<const TD*>(p.rowdec)[bi * p.dsb + hi * p.dsh + (int64_t)tt * p.dst])
                                 : 0.0f;
                }
                s_rowdec[r] = d;
            }
        }
        if constexpr (K::CONV) {  // reset flags of rows wr0-kConvHalo .. wr0+R-1, for the conv's window
            if (lane < R + kConvHalo) {
                const int t = t0 + wr0 - kConvHalo + lane;
                uint8_t rs = 0;
                if (p.seg != nullptr && t >= 0 && t < p.T) rs = p.seg[bi * p.sgb + (int64_t)t * p.sgt] != 0;
                base[K::OFF_CRESET + warp * 32 + lane] = rs;
            }
        }
        __syncwarp();
        ConvTaps ct;
        if constexpr (K::CONV) conv_taps<K>(p, v, c0, ct);  // in flight while the rows land
        PS dsp[4];  // SSD: the epilogue's D for this lane's channels, loaded while the rows land
        if constexpr (K::FORM == FORM_SSD) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int ca = c0 + chan<SPLIT>(2 * i, v), cb = c0 + chan<SPLIT>(2 * i + 1, v);
                dsp[i] = OS::pack(ca < p.C ? p.dskip[ca] : 0.0f, cb < p.C ? p.dskip[cb] : 0.0f);
            }
        }
        if (nvalid > wr0 && !mbar_wait_bounded(&s_bar[warp], par, kTmaPolls)) {
            atomicOr(&p.hdr[WS_ERROR], ERR_TMA);
            mbar_wait_bounded(&s_bar[warp], par, kTmaPolls);
        }
        if constexpr (K::CONV) {
            if (nvalid > wr0) conv_fold<K>(p, base, warp, q, v, wr0, ct);  // warp-uniform
        }

        // shared-memory row of virtual row r (REV: mirrored inside this warp's rows)
        auto srow = [&](int r) { return REV ? 2 * wr0 + R - 1 - r : r; };

        // ---------------------------------------------------------- phase 1
        // a, b of row r as 4 fp32 pairs (channels 2i, 2i+1 of this lane's vector);
        // `write` stores the rounded a, b back for phase 2.
        auto gates = [&](int r, bool write, float2 (&a)[4], float2 (&b)[4]) {
            const bool reset = s_reset[r] != 0;
            if constexpr (K::FORM == FORM_AFFINE || K::FORM == FORM_RETENTION) {
                if constexpr (K::ROWDEC) {
                    const float d = reset ? 0.0f : s_rowdec[r];
#pragma unroll
                    for (int i = 0; i < 4; ++i) a[i] = splat2(d);
                } else {
                    typename Ops<TD>::P dp[4];
                    Row8<TD, SPLIT>::lds(reinterpret_cast<const TD*>(slot_ptr<K>(base, 0)) + srow(r) * CBW, v, dp);
#pragma unroll
                    for (int i = 0; i < 4; ++i) a[i] = widen(dp[i]);
                    if (reset) {  // uniform across the row group
#pragma unroll
                        for (int i = 0; i < 4; ++i) a[i] = splat2(0.0f);
                    }
                }
                PS up[4];
                Row8<TS, SPLIT>::lds(reinterpret_cast<const TS*>(slot_ptr<K>(base, K::HAS_DSTREAM ? 1 : 0)) + srow(r) * CBW, v, up);
#pragma unroll
                for (int i = 0; i < 4; ++i) b[i] = widen(up[i]);
            } else {
                // GATED: slots z, g, x.  SSD: slots dt, bg, u (cg, og used in phase 2)
                TS* s0 = reinterpret_cast<TS*>(slot_ptr<K>(base, 0)) + srow(r) * CBW;
                TS* s1 = reinterpret_cast<TS*>(slot_ptr<K>(base, 1)) + srow(r) * CBW;
                TS* s2 = reinterpret_cast<TS*>(slot_ptr<K>(base, 2)) + srow(r) * CBW;
                PS p0[4], p1[4], p2[4], ap[4], bp[4];
                constexpr bool FIXB = FIX && K::FORM == FORM_GATED;  // slot 2 holds b itself
                Row8<TS, SPLIT>::lds(s0, v, p0);
                if constexpr (!FIXB) Row8<TS, SPLIT>::lds(s1, v, p1);
                Row8<TS, SPLIT>::lds(s2, v, p2);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    float2 dec;
                    if constexpr (K::FORM == FORM_GATED) {
                        dec = sig2<TS>(widen(p0[i]));
                    } else {
                        // need_kernels.py:330-332: fp32 dt = dt_min + scale * sigmoid(dt_raw)
                        // (separately rounded), decay = exp(-dt) rounded to the input dtype
                        const float2 dt = fadd2(fmul2(sig2<TS>(widen(p0[i])), splat2(p.dt_scale)), splat2(p.dt_min));
                        dec = exp2_pair<TS>(make_float2(-dt.x, -dt.y));
                    }
                    ap[i] = OS::pack(dec.x, dec.y);
                    if constexpr (FIXB) {
                        bp[i] = p2[i];
                    } else {
                        const float2 g = sig2<TS>(widen(p1[i]));
                        bp[i] = OS::mul(OS::sub(OS::one(), ap[i]), OS::mul(OS::pack(g.x, g.y), p2[i]));
                    }
                }
                if (reset) {  // uniform across the row group: one branch per row
#pragma unroll
                    for (int i = 0; i < 4; ++i) ap[i] = OS::zero();
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    a[i] = widen(ap[i]);
                    b[i] = widen(bp[i]);
                }
                if (write) {
                    Row8<TS, SPLIT>::sts(s0, v, ap);  // a over the decay input
                    if constexpr (K::FORM == FORM_GATED) Row8<TS, SPLIT>::sts(s2, v, bp);  // b over x
                    else Row8<TS, SPLIT>::sts(s1, v, bp);  // b over b_gate
                }
            }
        };
        // a, b written back by phase 1
        auto reload = [&](int r, float2 (&a)[4], float2 (&b)[4]) {
            if constexpr (K::FORM == FORM_AFFINE || K::FORM == FORM_RETENTION) {
                gates(r, false, a, b);
            } else {
                PS ap[4], bp[4];
                Row8<TS, SPLIT>::lds(reinterpret_cast<const TS*>(slot_ptr<K>(base, 0)) + srow(r) * CBW, v, ap);
                Row8<TS, SPLIT>::lds(reinterpret_cast<const TS*>(slot_ptr<K>(base, K::FORM == FORM_GATED ? 2 : 1)) + srow(r) * CBW, v, bp);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    a[i] = widen(ap[i]);
                    b[i] = widen(bp[i]);
                }
            }
        };

        float2 A[4], B[4];  // this thread's map, channel pairs
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            A[i] = splat2(1.0f);
            B[i] = splat2(0.0f);
        }
#pragma unroll kPhase1Unroll
        for (int j = 0; j < rend; ++j) {  // rows past T act as the identity
            float2 a[4], b[4];
            gates(r0 + j, true, a, b);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                B[i] = ffma2(a[i], B[i], b[i]);
                A[i] = fmul2(a[i], A[i]);
            }
        }
        // ---------------------------------------------------------- in-warp prefix
        // The row groups q of a warp hold consecutive rows: their inclusive maps
        // (rows of groups 0..q) by a Kogge-Stone scan over shuffles, and the
        // exclusive one (the rows before this thread's) from the group before.
#pragma unroll
        for (int d = 1; d < SS; d *= 2) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 oA = make_float2(__shfl_up_sync(0xffffffffu, A[i].x, d * LPR),
                                              __shfl_up_sync(0xffffffffu, A[i].y, d * LPR));
                const float2 oB = make_float2(__shfl_up_sync(0xffffffffu, B[i].x, d * LPR),
                                              __shfl_up_sync(0xffffffffu, B[i].y, d * LPR));
                if (q >= d) {
                    B[i] = ffma2(A[i], oB, B[i]);
                    A[i] = fmul2(A[i], oA);
                }
            }
        }
        float2 EA[4], EB[4];  // map of the warp's rows before this thread's rows
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 pA = make_float2(__shfl_up_sync(0xffffffffu, A[i].x, LPR), __shfl_up_sync(0xffffffffu, A[i].y, LPR));
            const float2 pB = make_float2(__shfl_up_sync(0xffffffffu, B[i].x, LPR), __shfl_up_sync(0xffffffffu, B[i].y, LPR));
            EA[i] = q > 0 ? pA : splat2(1.0f);
            EB[i] = q > 0 ? pB : splat2(0.0f);
        }
        // every lane's inclusive map; the last group's is the warp total the look-back warp reads
        if constexpr (K::AGG_SLOT >= 0) __syncwarp();  // every lane is done with the slot rows the map overwrites
#pragma unroll
        for (int i = 0; i < 4; ++i) agg4(warp)[i * 32 + lane] = make_float4(A[i].x, A[i].y, B[i].x, B[i].y);
        mbar_arrive(s_p1);
        named_sync(1, K::NT);  // the look-back warp has put this warp's entering state in s_hin

        // ---------------------------------------------------------- phase 2
        const bool run_phase2 = !DEFER || *s_defer == 0u;
        if constexpr (DEFER) {
            if (!run_phase2) {
                // a deferred tile: its rounded updates b (slot 2, written by phase 1)
                // go to its output rows, where the fix-up reads them back
                TS* brow = reinterpret_cast<TS*>(p.out) + bi * p.osb + hi * p.osh + (int64_t)(t0 + r0) * p.ost + c0;
                const bool okb0 = c0 + chan<SPLIT>(0, v) < p.C, okb1 = c0 + chan<SPLIT>(4, v) < p.C;
                for (int j = 0; j < rend; ++j, brow += p.ost) {
                    PS bq[4];
                    Row8<TS, SPLIT>::lds(reinterpret_cast<const TS*>(slot_ptr<K>(base, 2)) + (r0 + j) * CBW, v, bq);
                    Row8<TS, SPLIT>::stg(brow, v, bq, okb0, okb1);
                }
            }
        }
        if (run_phase2) {  // else the sequence-parallel fix-up writes this tile
        float2 h[4];
        {
            const float4 h0 = *reinterpret_cast<const float4*>(s_hin + warp * CBW + chan<SPLIT>(0, v));
            const float4 h1 = *reinterpret_cast<const float4*>(s_hin + warp * CBW + chan<SPLIT>(4, v));
            h[0] = ffma2(EA[0], make_float2(h0.x, h0.y), EB[0]);
            h[1] = ffma2(EA[1], make_float2(h0.z, h0.w), EB[1]);
            h[2] = ffma2(EA[2], make_float2(h1.x, h1.y), EB[2]);
            h[3] = ffma2(EA[3], make_float2(h1.z, h1.w), EB[3]);
        }
        const bool ok0 = c0 + chan<SPLIT>(0, v) < p.C;
        const bool ok1 = c0 + chan<SPLIT>(4, v) < p.C;
        const int64_t ostep = REV ? -p.ost : p.ost;  // REV: rows are written in decreasing t
        TS* orow = reinterpret_cast<TS*>(p.out) + bi * p.osb + hi * p.osh +
                   (int64_t)(REV ? p.T - 1 - t0 - r0 : t0 + r0) * p.ost + c0;
        // output row r: advances the state and forms the epilogue in o
        auto step = [&](int r, PS (&o)[4]) {
            float2 a[4], b[4];
            reload(r, a, b);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                h[i] = ffma2(a[i], h[i], b[i]);
                o[i] = OS::pack(h[i].x, h[i].y);  // state in the input dtype
            }
            if constexpr (K::FORM == FORM_SSD) {
                PS up[4], cp[4], gp[4];
                Row8<TS, SPLIT>::lds(reinterpret_cast<const TS*>(slot_ptr<K>(base, 2)) + srow(r) * CBW, v, up);
                Row8<TS, SPLIT>::lds(reinterpret_cast<const TS*>(slot_ptr<K>(base, 3)) + srow(r) * CBW, v, cp);
                Row8<TS, SPLIT>::lds(reinterpret_cast<const TS*>(slot_ptr<K>(base, 4)) + srow(r) * CBW, v, gp);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float2 cgs = sig2<TS>(widen(cp[i]));
                    const float2 ogs = sig2<TS>(widen(gp[i]));
                    // (cg * state + D * u) * og, each op in the input dtype
                    o[i] = OS::mul(OS::add(OS::mul(OS::pack(cgs.x, cgs.y), o[i]), OS::mul(dsp[i], up[i])),
                                   OS::pack(ogs.x, ogs.y));
                }
            } else if constexpr (K::FORM == FORM_RETENTION) {
                PS qp[4];
                Row8<TS, SPLIT>::lds(reinterpret_cast<const TS*>(slot_ptr<K>(base, K::HAS_DSTREAM ? 2 : 1)) + srow(r) * CBW, v, qp);
#pragma unroll
                for (int i = 0; i < 4; ++i) o[i] = OS::mul(qp[i], o[i]);
            }
        };
#pragma unroll kPhase2Unroll
        for (int j = 0; j < rend; ++j, orow += ostep) {
            PS o[4];
            step(r0 + j, o);
            Row8<TS, SPLIT>::stg(orow, v, o, ok0, ok1);
        }
        }  // phase 2
        }  // row warps
        if constexpr (FIX) {  // the stage is refilled by the next tile's TMA
            fence_proxy_async_shared();
            __syncthreads();
        }
    }  // tiles
}

}  // namespace need
