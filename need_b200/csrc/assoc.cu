// assoc.cu -- NEED's matrix-state associative memory on sm_100a tensor cores.
//
// HierarchicalMemory._linear_associative_memory (need_core.py:1960-2001) keeps,
// per sequence, a state S_t = sum_{s<=t} k_s (x) v_s [r, d] and z_t = sum k_s
// [r] over feature-mapped keys k = elu(k_raw) + 1, and reads
//     out_t = (q_t . S_t) / max(q_t . z_t, eps)      q = elu(q_raw) + 1.
// The reference materialises S_t for every token of a 32-token chunk.  Here a
// CTA owns a segment of one sequence and 128 columns of d and walks the
// segment in tiles of 128 tokens with the chunked (linear-attention) form,
// every product on tcgen05 tensor cores with fp32 accumulators in tensor memory:
//     P   = Q K^T                 (128 x 128, masked to s <= t)    TMEM cols   0..127
//     O   = P V + Q S             (128 tokens x 128 columns)       TMEM cols 128..255
//     S^T += V^T K                (128 columns x 64 features)      TMEM cols 256..319
// with the denominator q_t . z + sum_{s<=t} P[t, s] in fp32 on the CUDA cores.
// The state stays in tensor memory in fp32 for the whole segment; its bf16
// copy in shared memory is the B operand of the next tile's Q S.  A later
// segment starts from the state of the tiles before it: re-summed state-only
// in the same kernel, or summed once per chunk by assoc_state_kernel
// (assoc_plan picks the cheaper).
//
// Operands arrive by TMA with the 128-byte swizzle (no multicast); every tile
// is a canonical UMMA layout (umma.cuh), so the same shared-memory tile of V
// serves as the MN-major B of P V and the MN-major A of V^T K, and the tile of
// K as the K-major B of Q K^T and the MN-major B of V^T K.  Loads of the next
// tile overlap the current one (two stages); outputs leave through a TMA store.
//
// A prologue kernel applies the feature map (and the optional write mask) and
// writes q, k as bf16 [B, T, 64] (features past r zero) into the workspace;
// the chunk states, when the plan has them, follow in the same workspace.
#include <algorithm>
#include <atomic>
#include <climits>

#include "host_common.h"
#include "need_scan.h"
#include "ptx.cuh"
#include "scan_kernel.cuh"
#include "umma.cuh"

using namespace need;

namespace {

constexpr int kTok = 128;    // tokens per tile
constexpr int kCols = 128;   // columns of d per CTA
constexpr int kRank = 64;    // feature rank, zero padded
constexpr int kThreads = 256;  // two warpgroups
constexpr int kMainThreads = kThreads + 32;  // and, in the main kernel, one warp that issues the MMAs
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAssocPolls = 1u << 20;  // try_wait polls per wait before giving up

// shared memory map (offsets from a 1024-byte aligned base)
constexpr int OFF_Q = 0;                       // 2 stages x [128 tokens][64 features] bf16
constexpr int OFF_K = OFF_Q + 2 * 16384;       // 2 stages x [128 tokens][64 features]
constexpr int OFF_V = OFF_K + 2 * 16384;       // 2 stages x 2 boxes x [128 tokens][64 columns]
constexpr int OFF_P = OFF_V + 2 * 32768;       // 2 K-atoms x [128 tokens][64 tokens]
constexpr int OFF_S = OFF_P + 32768;           // [128 columns][64 features] (K-major B of Q S)
constexpr int OFF_O = OFF_S + 16384;           // 2 boxes x [128 tokens][64 columns], TMA store source
constexpr int OFF_Z = OFF_O + 32768;           // z [64], column sums [4][64], q.z [2 tiles][2][128], row sums [2][128] (fp32)
constexpr int OFF_BAR = OFF_Z + (5 * kRank + 6 * kTok) * 4;  // full[2], pbar, obar, tmem base
constexpr int SMEM_BYTES = OFF_BAR + 64 + 1024;  // + alignment slack

#ifndef NEED_ASSOC_MAX_SEG
#define NEED_ASSOC_MAX_SEG 24
#endif
constexpr int kMaxSeg = NEED_ASSOC_MAX_SEG;  // segments per sequence
constexpr int kMaxChunk = 64;  // state chunks per sequence
constexpr int kScanAbove = 4;  // more chunks than this: prefix-summed by a kernel of their own

struct AssocParams {
    CUtensorMap tm_q, tm_k, tm_v, tm_out;  // 3-D maps (column, token, sequence), 64 x 128 boxes, 128-byte swizzle
    int32_t T, d;
    float eps;
    uint32_t* hdr;  // workspace header: error word
    float* cs;      // chunk states [chunk][sequence][column block][128 columns][64 features] fp32
    float* cz;      // chunk feature sums [chunk][sequence][64] fp32
    int32_t nb, ncb;
    int32_t kchunk;   // chunks per segment before the last
    int32_t scanned;  // cs / cz hold running sums over the chunks (else each chunk's own)
    int32_t recompute;  // a later segment sums the tiles before it itself (no chunk states)
    int32_t seg[kMaxSeg + 1];      // segment s owns tiles seg[s] .. seg[s + 1] - 1
    int32_t chunk[kMaxChunk + 1];  // chunk c sums tiles chunk[c] .. chunk[c + 1] - 1
};

// z += column sums of a tile's k (bf16 [128 tokens][64 features], 128-byte
// swizzle): threads c, c + 64, c + 128, c + 192 each sum a quarter of the rows
// of feature c, thread c adds them to z[c] (call after every thread has read z)
__device__ __forceinline__ void add_z(const unsigned char* krow, float* z, float* zpart, int tid) {
    const int c = tid & 63, r0 = (tid >> 6) * 32;
    const int j = c >> 3, e = c & 7;
    float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 8
    for (int r = 0; r < 32; ++r) {
        const uint16_t hv = *reinterpret_cast<const uint16_t*>(krow + umma::sw128(r0 + r, j) + 2 * e);
        a[r & 3] += __uint_as_float(static_cast<uint32_t>(hv) << 16);
    }
    zpart[(tid >> 6) * kRank + c] = (a[0] + a[1]) + (a[2] + a[3]);
    named_sync(1, 256);
    if (tid < kRank) z[c] += (zpart[c] + zpart[kRank + c]) + (zpart[2 * kRank + c] + zpart[3 * kRank + c]);
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    const __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&p);
}

// ------------------------------------------------------------------ main kernel
// Grid (column blocks, sequences, segments).  Segment s owns tiles [seg[s],
// seg[s+1]).  A later segment starts from the state of the tiles before it:
// the sum, in chunk order, of the chunk states that assoc_state_kernel left in
// the workspace (or the running sum at its last chunk, after the chunk scan).
// Two warpgroups run the CUDA-core work.  Warp w reads tensor-memory lanes
// 32 (w % 4) .. + 31, so row (token, or column of d for the state) `row` =
// 32 (w % 4) + lane belongs to warps w and w + 4; warpgroup g takes half of each
// epilogue's columns.  A ninth warp issues the MMAs: an issuing thread stalls
// while the tensor pipe drains, and the warpgroups' column sums and the next
// tile's q.z run meanwhile.
__global__ void __launch_bounds__(kMainThreads, 1) assoc_kernel(const __grid_constant__ AssocParams p) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* base =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* z = reinterpret_cast<float*>(base + OFF_Z);  // [64] sum of k over the tiles so far
    float* zpart = z + kRank;                           // [4][64] column sums of a quarter of the rows
    float* s_qz = zpart + 4 * kRank;                    // [2 tiles][2][128] q_t . z, per half of the features
    float* s_rs = s_qz + 4 * kTok;                      // [2][128] masked row sums of P, per half
    uint64_t* full = reinterpret_cast<uint64_t*>(base + OFF_BAR);  // [2] tile loads
    uint64_t* pbar = full + 2;  // P = Q K^T done
    uint64_t* obar = full + 3;  // O and the state update done
    uint32_t* tbase = reinterpret_cast<uint32_t*>(full + 4);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int wg = warp >> 2, lw = warp & 3;
    const int row = lw * 32 + lane;
    const bool compute = warp < kThreads / 32, mma_thread = tid == kThreads;
    const int c0 = blockIdx.x * kCols, b = blockIdx.y;
    const int start = p.seg[blockIdx.z];  // this CTA's first own tile
    const int end = p.seg[blockIdx.z + 1];
    if (start >= end) return;  // no tiles (before any allocation or barrier)
    const uint32_t sbase = smem_addr(base);

    if (tid == 0) {
        mbar_init(&full[0], 1);
        mbar_init(&full[1], 1);
        mbar_init(pbar, 1);
        mbar_init(obar, 1);
        fence_barrier_init();
    }
    if (tid < kRank) z[tid] = 0.0f;
    if (warp == 0) {
        umma::tmem_alloc(tbase, kTmemCols);
        umma::tmem_relinquish();
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = *tbase;
    const uint32_t lane_off = static_cast<uint32_t>(lw * 32) << 16;  // this warp's TMEM lanes
    const uint32_t tP = tmem + lane_off, tO = tmem + 128 + lane_off, tS = tmem + 256 + lane_off;
    const uint32_t dP = tmem, dO = tmem + 128, dS = tmem + 256;  // MMA destinations

    constexpr uint32_t ID_QK = umma::idesc_bf16(128, 128, umma::K_MAJOR, umma::K_MAJOR);
    constexpr uint32_t ID_PV = umma::idesc_bf16(128, 128, umma::K_MAJOR, umma::MN_MAJOR);
    constexpr uint32_t ID_QS = umma::idesc_bf16(128, 128, umma::K_MAJOR, umma::K_MAJOR);
    constexpr uint32_t ID_VK = umma::idesc_bf16(128, 64, umma::MN_MAJOR, umma::MN_MAJOR);

    // Own tile `it` sits in stage (it - start) & 1.  fpar holds the phase each
    // stage's barrier completes next; pend (thread 0) the stages with a load in flight.
    uint32_t fpar = 0, pend = 0;
    auto own_stage = [&](int it) { return (it - start) & 1; };
    auto issue_own = [&](int tile) {
        const int st = own_stage(tile), t0 = tile * kTok;
        pend |= 1u << st;
        mbar_arrive_expect_tx(&full[st], 16384u + 16384u + 32768u);
        umma::tma_load_3d(base + OFF_Q + st * 16384, &p.tm_q, 0, t0, b, &full[st]);
        umma::tma_load_3d(base + OFF_K + st * 16384, &p.tm_k, 0, t0, b, &full[st]);
        umma::tma_load_3d(base + OFF_V + st * 32768, &p.tm_v, c0, t0, b, &full[st]);
        umma::tma_load_3d(base + OFF_V + st * 32768 + 16384, &p.tm_v, c0 + 64, t0, b, &full[st]);  // may lie past d
    };
    // With p.recompute a later segment first runs the tiles before it
    // state-only, two per step: step j holds tiles 2j and 2j + 1 in stage j & 1,
    // the first in the stage's K / V slots, the second in P (K) and O or Q (V),
    // buffers that this mode leaves idle.
    const int nsteps = p.recompute ? (start + 1) >> 1 : 0;
    auto pre_k = [](int st, int h) { return h == 0 ? OFF_K + st * 16384 : OFF_P + st * 16384; };
    auto pre_v = [](int st, int h) { return h == 0 ? OFF_V + st * 32768 : (st == 0 ? OFF_O : OFF_Q); };
    auto issue_pre = [&](int j) {
        const int st = j & 1, n = min(2, start - 2 * j);
        pend |= 1u << st;
        mbar_arrive_expect_tx(&full[st], static_cast<uint32_t>(n) * (16384u + 32768u));
        for (int h = 0; h < n; ++h) {
            const int t0 = (2 * j + h) * kTok;
            umma::tma_load_3d(base + pre_k(st, h), &p.tm_k, 0, t0, b, &full[st]);
            umma::tma_load_3d(base + pre_v(st, h), &p.tm_v, c0, t0, b, &full[st]);
            umma::tma_load_3d(base + pre_v(st, h) + 16384, &p.tm_v, c0 + 64, t0, b, &full[st]);
        }
    };
    if (tid == 0) {
        if (nsteps > 0) {
            issue_pre(0);
            if (nsteps > 1) issue_pre(1);
        } else {
            issue_own(start);
            if (start + 1 < end) issue_own(start + 1);
        }
    }

    bool ok = true;
    uint32_t pph = 0, oph = 0;  // phases of the P barrier and the O / state barrier
    auto wait_full = [&](int st) {  // a stage's loads, by every thread
        const bool got = mbar_wait_bounded(&full[st], (fpar >> st) & 1u, kAssocPolls);
        ok &= got;
        if (got) fpar ^= 1u << st, pend &= ~(1u << st);
    };
    bool qk_ahead = false;  // the MMA thread: the next tile's P is issued already
    auto issue_qk = [&](int tile) {  // P = Q K^T of `tile`, whose loads have landed
        const int st = own_stage(tile);
        const uint32_t sQ = sbase + OFF_Q + st * 16384, sK = sbase + OFF_K + st * 16384;
        umma::fence_after_sync();
#pragma unroll
        for (int k = 0; k < kRank / 16; ++k)
            umma::mma_bf16(dP, umma::smem_desc(sQ + 32 * k, 16, 1024), umma::smem_desc(sK + 32 * k, 16, 1024), ID_QK,
                           k > 0);
        umma::mma_commit(pbar);
    };
    auto store_row_chunks = [&](unsigned char* dst, int r, int j0, const uint32_t (&pk)[16]) {
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4)
            *reinterpret_cast<uint4*>(dst + umma::sw128(r, j0 + q4)) =
                make_uint4(pk[4 * q4], pk[4 * q4 + 1], pk[4 * q4 + 2], pk[4 * q4 + 3]);
    };
    // the bf16 copy of the state in TMEM, as the K-major B of the next Q S (row =
    // column of d; this warpgroup's 32 features)
    auto copy_state = [&]() {
        float v[32];
        umma::tmem_ld32(tS + 32 * wg, v);
        umma::tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) pk[e / 2] = pack_bf16(v[e], v[e + 1]);
        store_row_chunks(base + OFF_S, row, wg * 4, pk);
    };

    int aborted_at = -1;
    // ---- state-only tiles before this CTA's segment, two per step
    for (int j = 0; j < nsteps; ++j) {
        const int st = j & 1, n = min(2, start - 2 * j);
        wait_full(st);
        if (mma_thread) {
            umma::fence_after_sync();
            for (int h = 0; h < n; ++h) {
                const uint32_t sK = sbase + pre_k(st, h), sV = sbase + pre_v(st, h);
#pragma unroll
                for (int k = 0; k < kTok / 16; ++k)
                    umma::mma_bf16(dS, umma::smem_desc(sV + 2048 * k, 16384, 1024),
                                   umma::smem_desc(sK + 2048 * k, 16384, 1024), ID_VK, j > 0 || h > 0 || k > 0);
            }
            umma::mma_commit(obar);
        }
        if (compute) {
            add_z(base + pre_k(st, 0), z, zpart, tid);
            if (n > 1) {
                named_sync(1, kThreads);  // the first tile's column sums are read
                add_z(base + pre_k(st, 1), z, zpart, tid);
            }
        }
        ok &= mbar_wait_bounded(obar, oph, kAssocPolls);
        oph ^= 1u;
        umma::fence_after_sync();
        umma::fence_before_sync();
        if (!__syncthreads_and(ok)) {
            aborted_at = 2 * j;
            break;
        }
        if (tid == 0 && j + 2 < nsteps) issue_pre(j + 2);  // the stage's MMAs and readers are done
    }
    if (nsteps > 0 && aborted_at < 0) {  // the state entering the segment, for its first Q S
        if (tid == 0) {  // every buffer of the state-only steps is free now
            issue_own(start);
            if (start + 1 < end) issue_own(start + 1);
        }
        if (compute) copy_state();
        fence_proxy_async_shared();
        umma::fence_before_sync();
        __syncthreads();
    }
    if (start > 0 && !p.recompute && compute) {  // the state entering the segment: chunk sums in chunk order
        const int chi = static_cast<int>(blockIdx.z) * p.kchunk, clo = p.scanned ? chi - 1 : 0;
        float acc[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) acc[e] = 0.0f;
        for (int c = clo; c < chi; ++c) {
            const float4* src = reinterpret_cast<const float4*>(
                p.cs + ((static_cast<size_t>(c) * p.nb + b) * p.ncb + blockIdx.x) * (kCols * kRank) + row * kRank +
                32 * wg);
#pragma unroll
            for (int q4 = 0; q4 < 8; ++q4) {
                const float4 f = src[q4];
                acc[4 * q4] += f.x, acc[4 * q4 + 1] += f.y, acc[4 * q4 + 2] += f.z, acc[4 * q4 + 3] += f.w;
            }
        }
        umma::tmem_st32(tS + 32 * wg, acc);
        if (tid < kRank) {
            float zz = 0.0f;
            for (int c = clo; c < chi; ++c) zz += p.cz[(static_cast<size_t>(c) * p.nb + b) * kRank + tid];
            z[tid] = zz;
        }
        umma::tmem_wait_st();
    }
    if (start > 0 && !p.recompute) {
        umma::fence_before_sync();
        __syncthreads();
        umma::fence_after_sync();
        if (compute) copy_state();
        fence_proxy_async_shared();
        umma::fence_before_sync();
        __syncthreads();
    }
    // q_t . z over the tiles before `it`, this warpgroup's half of the features,
    // into the tile's q.z slot (its loads have landed)
    auto qdotz = [&](int it) {
        const unsigned char* qrow = base + OFF_Q + own_stage(it) * 16384;
        float qz0 = 0.0f, qz1 = 0.0f;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            const int j = 4 * wg + jj;
            const uint4 w = *reinterpret_cast<const uint4*>(qrow + umma::sw128(row, j));
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                qz0 = fmaf(__uint_as_float(ws[e] << 16), z[8 * j + 2 * e], qz0);
                qz1 = fmaf(__uint_as_float(ws[e] & 0xffff0000u), z[8 * j + 2 * e + 1], qz1);
            }
        }
        s_qz[((it - start) & 1) * 2 * kTok + wg * kTok + row] = qz0 + qz1;
    };
    if (aborted_at < 0 && start < end) {  // the first tile's loads, P and q.z
        wait_full(own_stage(start));
        if (mma_thread) {
            issue_qk(start);
            qk_ahead = true;
        }
        if (compute) qdotz(start);
    }
    // ---- own tiles.  Tile it: its P epilogue; its MMA group on the tensor
    // cores, with the next tile's Q K^T behind it, while the warpgroups add its
    // k to z and take the next tile's q.z; then its outputs and state copy.
    for (int it = start; it < end && aborted_at < 0; ++it) {
        const int st = own_stage(it), qs = (it - start) & 1;
        const bool next = it + 1 < end;
        const int t0 = it * kTok;
        const uint32_t sQ = sbase + OFF_Q + st * 16384, sK = sbase + OFF_K + st * 16384;
        const uint32_t sV = sbase + OFF_V + st * 32768;
        const uint32_t sP = sbase + OFF_P, sS = sbase + OFF_S;
        const unsigned char* krow = base + OFF_K + st * 16384;

        ok &= mbar_wait_bounded(pbar, pph, kAssocPolls);
        pph ^= 1u;
        qk_ahead = false;
        umma::fence_after_sync();

        // ---- P epilogue over this warpgroup's 64 columns: blocks of 32 source
        // tokens above the diagonal are all masked (no load), below it none are
        if (compute) {
            float rs = 0.0f;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int cb = 2 * wg + h;  // 32-column block
                uint32_t pk[16];
                if (cb > lw) {
#pragma unroll
                    for (int e = 0; e < 16; ++e) pk[e] = 0u;
                } else {
                    float v[32];
                    umma::tmem_ld32(tP + 32 * cb, v);
                    umma::tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 32; e += 2) {
                        const float a0 = (cb < lw || e <= lane) ? v[e] : 0.0f;
                        const float a1 = (cb < lw || e + 1 <= lane) ? v[e + 1] : 0.0f;
                        rs += a0 + a1;
                        pk[e / 2] = pack_bf16(a0, a1);
                    }
                }
                store_row_chunks(base + OFF_P + wg * 16384, row, h * 4, pk);
            }
            s_rs[wg * kTok + row] = rs;
        }
        fence_proxy_async_shared();  // P and last tile's state copy visible to the tensor cores
        if (tid == 0) umma::tma_store_wait_read();  // last tile's output store has left shared memory
        umma::fence_before_sync();
        __syncthreads();

        // ---- O = P V + Q S; S^T += V^T K; then the next tile's P (its TMEM
        // columns were read out above)
        if (mma_thread) {
            umma::fence_after_sync();
#pragma unroll
            for (int k = 0; k < kTok / 16; ++k)
                umma::mma_bf16(dO, umma::smem_desc(sP + (k >> 2) * 16384 + 32 * (k & 3), 16, 1024),
                               umma::smem_desc(sV + 2048 * k, 16384, 1024), ID_PV, k > 0);
            if (it > 0) {
#pragma unroll
                for (int k = 0; k < kRank / 16; ++k)
                    umma::mma_bf16(dO, umma::smem_desc(sQ + 32 * k, 16, 1024), umma::smem_desc(sS + 32 * k, 16, 1024),
                                   ID_QS, true);
            }
#pragma unroll
            for (int k = 0; k < kTok / 16; ++k)
                umma::mma_bf16(dS, umma::smem_desc(sV + 2048 * k, 16384, 1024),
                               umma::smem_desc(sK + 2048 * k, 16384, 1024), ID_VK, it > 0 || k > 0);
            umma::mma_commit(obar);
            if (next) {
                const int nx = own_stage(it + 1);
                ok &= mbar_wait_bounded(&full[nx], (fpar >> nx) & 1u, kAssocPolls);  // ahead of wait_full
                issue_qk(it + 1);
                qk_ahead = true;
            }
        }
        if (compute) {
            add_z(krow, z, zpart, tid);
            named_sync(1, kThreads);  // z with this tile, for the next q.z
        }
        if (next) {
            wait_full(own_stage(it + 1));
            if (compute) qdotz(it + 1);
        }
        ok &= mbar_wait_bounded(obar, oph, kAssocPolls);
        oph ^= 1u;
        umma::fence_after_sync();
        // every reader of this stage is done (the MMAs by the barrier, q.z and
        // the column sums before the barriers above): refill it now
        if (tid == 0 && it + 2 < end) issue_own(it + 2);

        // ---- outputs: O / max(q.z + rowsum, eps) in bf16, this warpgroup's 64
        // columns (one TMA store box), staged for the store; then the state
        // after this tile, for the next tile's Q S
        if (compute) {
            const float* qz = s_qz + qs * 2 * kTok;
            const float den = (qz[row] + qz[kTok + row]) + (s_rs[row] + s_rs[kTok + row]);
            const float inv = 1.0f / fmaxf(den, p.eps);
            float v[2][32];
            umma::tmem_ld32(tO + 64 * wg, v[0]);
            umma::tmem_ld32(tO + 64 * wg + 32, v[1]);
            umma::tmem_wait_ld();
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                uint32_t pk[16];
#pragma unroll
                for (int e = 0; e < 32; e += 2) pk[e / 2] = pack_bf16(v[h][e] * inv, v[h][e + 1] * inv);
                store_row_chunks(base + OFF_O + wg * 16384, row, h * 4, pk);
            }
            if (next) copy_state();
        }
        fence_proxy_async_shared();  // staged outputs (TMA store) and S (next MMA) visible to the async proxy
        umma::fence_before_sync();
        if (!__syncthreads_and(ok)) {  // a wait gave up: stop (uniformly) and report
            aborted_at = it;
            break;
        }
        if (tid == 0) {
            umma::tma_store_3d(&p.tm_out, base + OFF_O, c0, t0, b);
            if (c0 + 64 < p.d) umma::tma_store_3d(&p.tm_out, base + OFF_O + 16384, c0 + 64, t0, b);
            umma::tma_store_commit();
        }
    }
    // after a give-up, the next tile's P may still be in flight: its commit
    // covers every MMA issued, so wait (bounded) before freeing tensor memory
    if (mma_thread && aborted_at >= 0 && qk_ahead) mbar_wait_bounded(pbar, pph, kAssocPolls);
    if (tid == 0 && aborted_at >= 0) {  // loads still in flight land before the CTA exits
        for (int st = 0; st < 2; ++st)
            if (pend & (1u << st)) mbar_wait_bounded(&full[st], (fpar >> st) & 1u, kAssocPolls);
    }
    if (tid == 0) umma::tma_store_wait_all();
    if (!ok) atomicOr(&p.hdr[WS_ERROR], ERR_TMA);
    umma::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        umma::fence_after_sync();
        umma::tmem_dealloc(tmem, kTmemCols);
    }
}

// ------------------------------------------------------------------ chunk states
// Grid (column blocks, sequences, chunks).  A CTA sums its chunk's tiles:
// S^T = sum V^T K on the tensor cores (fp32 in tensor memory) and z = sum k;
// it writes them to cs / cz (z from column block 0 only: every block computes
// the same).  A ring of four K / V stages keeps three tiles' loads in flight
// while one is summed.
constexpr int kRing = 4;
constexpr int CS_OFF_K = 0;                         // 4 x [128 tokens][64 features] bf16
constexpr int CS_OFF_V = CS_OFF_K + kRing * 16384;  // 4 x 2 boxes x [128 tokens][64 columns]
constexpr int CS_OFF_Z = CS_OFF_V + kRing * 32768;  // z [64], column sums [4][64] (fp32)
constexpr int CS_OFF_BAR = CS_OFF_Z + 5 * kRank * 4;  // full[4], done, tmem base
constexpr int CS_SMEM_BYTES = CS_OFF_BAR + 64 + 1024;

__global__ void __launch_bounds__(kThreads, 1) assoc_state_kernel(const __grid_constant__ AssocParams p) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* base =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* z = reinterpret_cast<float*>(base + CS_OFF_Z);
    float* zpart = z + kRank;
    uint64_t* full = reinterpret_cast<uint64_t*>(base + CS_OFF_BAR);
    uint64_t* done = full + kRing;  // the tile's MMAs have read its stage
    uint32_t* tbase = reinterpret_cast<uint32_t*>(done + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int wg = warp >> 2, row = (warp & 3) * 32 + lane;
    const int cb = blockIdx.x, c0 = cb * kCols, b = blockIdx.y, chunk = blockIdx.z;
    const int t_lo = p.chunk[chunk], n = p.chunk[chunk + 1] - t_lo;
    if (n <= 0) return;
    const bool zsum = cb == 0;
    const uint32_t sbase = smem_addr(base);

    if (tid == 0) {
        for (int i = 0; i < kRing; ++i) mbar_init(&full[i], 1);
        mbar_init(done, 1);
        fence_barrier_init();
    }
    if (tid < kRank) z[tid] = 0.0f;
    if (warp == 0) {
        umma::tmem_alloc(tbase, 64);
        umma::tmem_relinquish();
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = *tbase;
    const uint32_t tS = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    constexpr uint32_t ID_VK = umma::idesc_bf16(128, 64, umma::MN_MAJOR, umma::MN_MAJOR);

    uint32_t fpar = 0, pend = 0;  // per stage: the phase completing next; a load in flight (thread 0)
    auto issue = [&](int i) {
        const int st = i % kRing, t0 = (t_lo + i) * kTok;
        pend |= 1u << st;
        mbar_arrive_expect_tx(&full[st], 16384u + 32768u);
        umma::tma_load_3d(base + CS_OFF_K + st * 16384, &p.tm_k, 0, t0, b, &full[st]);
        umma::tma_load_3d(base + CS_OFF_V + st * 32768, &p.tm_v, c0, t0, b, &full[st]);
        umma::tma_load_3d(base + CS_OFF_V + st * 32768 + 16384, &p.tm_v, c0 + 64, t0, b, &full[st]);
    };
    if (tid == 0)
        for (int i = 0; i < min(kRing, n); ++i) issue(i);

    bool ok = true;
    uint32_t dph = 0;
    int i = 0;
    for (; i < n; ++i) {
        const int st = i % kRing;
        const bool got = mbar_wait_bounded(&full[st], (fpar >> st) & 1u, kAssocPolls);
        ok &= got;
        if (got) fpar ^= 1u << st, pend &= ~(1u << st);
        if (tid == 0) {
            umma::fence_after_sync();
            const uint32_t sK = sbase + CS_OFF_K + st * 16384, sV = sbase + CS_OFF_V + st * 32768;
#pragma unroll
            for (int k = 0; k < kTok / 16; ++k)
                umma::mma_bf16(tmem, umma::smem_desc(sV + 2048 * k, 16384, 1024),
                               umma::smem_desc(sK + 2048 * k, 16384, 1024), ID_VK, i > 0 || k > 0);
            umma::mma_commit(done);
        }
        if (zsum) add_z(base + CS_OFF_K + st * 16384, z, zpart, tid);
        ok &= mbar_wait_bounded(done, dph, kAssocPolls);
        dph ^= 1u;
        umma::fence_after_sync();
        umma::fence_before_sync();
        if (!__syncthreads_and(ok)) break;
        if (tid == 0 && i + kRing < n) issue(i + kRing);  // the stage's MMAs and readers are done
    }
    if (i == n) {
        float v[32];
        umma::tmem_ld32(tS + 32 * wg, v);
        umma::tmem_wait_ld();
        float4* dst = reinterpret_cast<float4*>(
            p.cs + ((static_cast<size_t>(chunk) * p.nb + b) * p.ncb + cb) * (kCols * kRank) + row * kRank + 32 * wg);
#pragma unroll
        for (int q4 = 0; q4 < 8; ++q4) dst[q4] = make_float4(v[4 * q4], v[4 * q4 + 1], v[4 * q4 + 2], v[4 * q4 + 3]);
        if (zsum && tid < kRank) p.cz[(static_cast<size_t>(chunk) * p.nb + b) * kRank + tid] = z[tid];
    } else if (tid == 0) {  // a wait gave up: loads still in flight land before the CTA exits
        for (int st = 0; st < kRing; ++st)
            if (pend & (1u << st)) mbar_wait_bounded(&full[st], (fpar >> st) & 1u, kAssocPolls);
        atomicOr(&p.hdr[WS_ERROR], ERR_TMA);
    }
    umma::fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        umma::fence_after_sync();
        umma::tmem_dealloc(tmem, 64);
    }
}

// Running sums over the chunks, in place and in chunk order: cs[c] := cs[0] +
// ... + cs[c], the same for cz.  Thread i owns one float4 of every chunk; its
// loads go out sixteen chunks at a time.
__global__ void __launch_bounds__(256) assoc_chunk_scan_kernel(float* __restrict__ cs, float* __restrict__ cz,
                                                               int64_t cs4, int64_t cz4, int nchunk) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    float4* col;
    int64_t stride;
    if (i < cs4) col = reinterpret_cast<float4*>(cs) + i, stride = cs4;
    else if (i < cs4 + cz4) col = reinterpret_cast<float4*>(cz) + (i - cs4), stride = cz4;
    else return;
    constexpr int kBatch = 16;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);  // 0 + cs[0] is cs[0]: the main kernel's sums start so too
    for (int c0 = 0; c0 < nchunk; c0 += kBatch) {
        float4 f[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; ++j)
            if (c0 + j < nchunk) f[j] = __ldcg(col + (c0 + j) * stride);
#pragma unroll
        for (int j = 0; j < kBatch; ++j)
            if (c0 + j < nchunk) {
                acc.x += f[j].x, acc.y += f[j].y, acc.z += f[j].z, acc.w += f[j].w;
                col[(c0 + j) * stride] = acc;
            }
    }
}

// ------------------------------------------------------------------ feature map
// One warp per kFeatRows tokens: q, k -> bf16(elu(x) + 1) (need_core.py:1977-1978), zero past
// r; with a write mask w = bf16(clamp(mask, 0, 1)): k := bf16(k * w) and
// v := bf16(v * w) (need_core.py:1979-1984).
struct FeatArgs {
    const void* q;
    const void* k;
    int64_t qsb, qst, ksb, kst;
    int32_t qk32;  // q, k are fp32 (else bf16)
    int32_t pairs; // fp32 q, k with 8-byte aligned rows: each lane loads its two features at once
    const void* mask;
    int32_t mask32;
    int64_t msb, mst;
    const __nv_bfloat16* v;
    int64_t vsb, vst;
    __nv_bfloat16* qf;
    __nv_bfloat16* kf;
    __nv_bfloat16* vm;  // [nb, T, d] masked values, when mask
    int64_t nb, T, r, d;
};

__device__ __forceinline__ float ld_any(const void* base, int64_t i, bool f32) {
    return f32 ? static_cast<const float*>(base)[i] : __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i]);
}
// elu(x) + 1 before its rounding to bf16: x + 1 above 0, exp(x) = expm1(x) + 1
// at or below 0 (one hardware 2^x; its few-ulp fp32 error only moves the bf16
// result where the value lies within those ulp of a rounding tie)
__device__ __forceinline__ float feature_raw(float x) {
    float e;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(fminf(x, 0.0f) * 1.4426950408889634f));
    return x > 0.0f ? x + 1.0f : e;
}
__device__ __forceinline__ float rbf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

constexpr int kFeatRows = 4;  // rows per warp, their loads in flight together

__global__ void __launch_bounds__(128) assoc_features_kernel(const FeatArgs a) {
    const int lane = threadIdx.x & 31;
    const int64_t row0 = (static_cast<int64_t>(blockIdx.x) * 4 + (threadIdx.x >> 5)) * kFeatRows;
    const int64_t nrows = a.nb * a.T;
    // row -> (sequence, token) in 32 bits (the host limits nb * T below 2^31)
    const uint32_t T32 = static_cast<uint32_t>(a.T);
    const uint32_t b0 = static_cast<uint32_t>(row0) / T32, tt0 = static_cast<uint32_t>(row0) - b0 * T32;
    float qv[kFeatRows][2], kv[kFeatRows][2], w[kFeatRows];
#pragma unroll
    for (int i = 0; i < kFeatRows; ++i) {
        const int64_t row = row0 + i;
        uint32_t bu = b0, tu = tt0 + i;
        while (tu >= T32) tu -= T32, ++bu;  // at most kFeatRows steps
        const int64_t bi = bu, t = tu;
        w[i] = 1.0f;
        if (a.pairs) {
            const bool in = row < nrows && 2 * lane < a.r;
            const float2 qq = in ? *reinterpret_cast<const float2*>(static_cast<const float*>(a.q) + bi * a.qsb +
                                                                     t * a.qst + 2 * lane)
                                 : make_float2(0.0f, 0.0f);
            const float2 kk = in ? *reinterpret_cast<const float2*>(static_cast<const float*>(a.k) + bi * a.ksb +
                                                                     t * a.kst + 2 * lane)
                                 : make_float2(0.0f, 0.0f);
            qv[i][0] = qq.x, qv[i][1] = qq.y, kv[i][0] = kk.x, kv[i][1] = kk.y;
        } else {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int c = 2 * lane + e;
                const bool in = row < nrows && c < a.r;
                qv[i][e] = in ? ld_any(a.q, bi * a.qsb + t * a.qst + c, a.qk32) : 0.0f;
                kv[i][e] = in ? ld_any(a.k, bi * a.ksb + t * a.kst + c, a.qk32) : 0.0f;
            }
        }
        if (a.mask != nullptr && row < nrows) w[i] = ld_any(a.mask, bi * a.msb + t * a.mst, a.mask32);
    }
#pragma unroll
    for (int i = 0; i < kFeatRows; ++i) {
        const int64_t row = row0 + i;
        if (row >= nrows) break;
        const float wi = fminf(fmaxf(__bfloat162float(__float2bfloat16_rn(w[i])), 0.0f), 1.0f);
        float qf[2], kf[2];  // rounded to bf16 once, by the packing below
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const bool in = 2 * lane + e < a.r;
            qf[e] = in ? feature_raw(qv[i][e]) : 0.0f;
            kf[e] = in ? feature_raw(kv[i][e]) : 0.0f;
            if (a.mask != nullptr) kf[e] = rbf(rbf(kf[e]) * wi);
        }
        reinterpret_cast<uint32_t*>(a.qf + row * kRank)[lane] = pack_bf16(qf[0], qf[1]);
        reinterpret_cast<uint32_t*>(a.kf + row * kRank)[lane] = pack_bf16(kf[0], kf[1]);
        if (a.mask != nullptr) {
            uint32_t bu = b0, tu = tt0 + i;
            while (tu >= T32) tu -= T32, ++bu;
            const int64_t bi = bu, t = tu;
            const __nv_bfloat16* src = a.v + bi * a.vsb + t * a.vst;
            __nv_bfloat16* dst = a.vm + row * a.d;
            for (int64_t c = 8 * lane; c < a.d; c += 256) {
                const uint4 x = *reinterpret_cast<const uint4*>(src + c);
                const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
                uint32_t o[4];
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    o[k] = pack_bf16(__uint_as_float(xs[k] << 16) * wi, __uint_as_float(xs[k] & 0xffff0000u) * wi);
                *reinterpret_cast<uint4*>(dst + c) = make_uint4(o[0], o[1], o[2], o[3]);
            }
        }
    }
}

// ------------------------------------------------------------------ one-token step
// HierarchicalMemory.stream_step's associative memory (need_core.py:2067-2080)
// for one token of each sequence, every op in the model dtype TS as the
// reference rounds it: the state [r, d] and denominator [r] are updated in
// place, the output is (q . state) / max(q . denom, eps).  One CTA per
// sequence; thread i < r maps feature i, then each thread owns 16-byte column
// pieces and walks the r rows of the state.  The sums over features are taken
// in feature order with separately rounded fp32 products and adds.
constexpr int kStepThreads = 128;
constexpr int kStepMaxRank = 256;

struct StepParams {
    const void* q;
    const void* k;
    int64_t qs, ks;
    int32_t qk32;
    const void* v;
    int64_t vs;
    const void* mask;
    int32_t mask32;
    void* state;
    int64_t sn, sr;
    void* denom;
    int64_t dn;
    const int32_t* slot;
    void* out;
    int64_t os;
    int32_t r, d;
    float eps;
};

template <typename TS>
__device__ __forceinline__ float rnd_to(float x) {
    return to_f(static_cast<TS>(x));
}
template <>
__device__ __forceinline__ float rnd_to<float>(float x) {
    return x;
}

template <typename TS>
__global__ void __launch_bounds__(kStepThreads) assoc_step_kernel(const StepParams p) {
    using PS = typename Ops<TS>::P;
    constexpr int VEC = 16 / Ops<TS>::BYTES;
    __shared__ float s_q[kStepMaxRank], s_k[kStepMaxRank], s_dq[kStepMaxRank];
    __shared__ float s_w, s_den;
    const int n = blockIdx.x, tid = threadIdx.x;
    const int64_t slot = p.slot != nullptr ? p.slot[n] : n;
    TS* st = static_cast<TS*>(p.state) + slot * p.sn;
    TS* dn = static_cast<TS*>(p.denom) + slot * p.dn;
    const bool masked = p.mask != nullptr;
    const float w = masked ? fminf(fmaxf(rnd_to<TS>(ld_any(p.mask, n, p.mask32)), 0.0f), 1.0f) : 1.0f;
    for (int i = tid; i < p.r; i += kStepThreads) {
        const float qv = ld_any(p.q, n * p.qs + i, p.qk32), kv = ld_any(p.k, n * p.ks + i, p.qk32);
        const float qf = rnd_to<TS>((qv > 0.0f ? qv : expm1f(qv)) + 1.0f);
        float kf = rnd_to<TS>((kv > 0.0f ? kv : expm1f(kv)) + 1.0f);
        if (masked) kf = rnd_to<TS>(__fmul_rn(kf, w));
        const float d_new = rnd_to<TS>(__fadd_rn(to_f(dn[i]), kf));
        dn[i] = static_cast<TS>(d_new);
        s_q[i] = qf;
        s_k[i] = kf;
        s_dq[i] = rnd_to<TS>(__fmul_rn(qf, d_new));
    }
    if (tid == 0) s_w = w;
    __syncthreads();
    if (tid == 0) {
        float den = 0.0f;
        for (int i = 0; i < p.r; ++i) den = __fadd_rn(den, s_dq[i]);
        s_den = fmaxf(rnd_to<TS>(den), rnd_to<TS>(p.eps));
    }
    __syncthreads();
    const float den = s_den;
    const TS* v = static_cast<const TS*>(p.v) + n * p.vs;
    TS* out = static_cast<TS*>(p.out) + n * p.os;
    for (int c = tid * VEC; c < p.d; c += kStepThreads * VEC) {
        float vv[VEC], acc[VEC];
        {
            const uint4 u = *reinterpret_cast<const uint4*>(v + c);
            const PS* h = reinterpret_cast<const PS*>(&u);
#pragma unroll
            for (int e = 0; e < VEC / 2; ++e) {
                const float2 f = widen(h[e]);
                vv[2 * e] = masked ? rnd_to<TS>(__fmul_rn(f.x, w)) : f.x;
                vv[2 * e + 1] = masked ? rnd_to<TS>(__fmul_rn(f.y, w)) : f.y;
            }
        }
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[e] = 0.0f;
        // rows in batches of U, in row order; the next batch's loads are issued
        // before this batch is updated and stored, so one batch is always in flight
        constexpr int U = 8;
        auto load = [&](uint4 (&u)[U], int i0) {
#pragma unroll
            for (int k = 0; k < U; ++k)
                if (i0 + k < p.r) u[k] = *reinterpret_cast<const uint4*>(st + (int64_t)(i0 + k) * p.sr + c);
        };
        auto update = [&](uint4 (&u)[U], int i0) {
#pragma unroll
            for (int k = 0; k < U; ++k) {
                const int i = i0 + k;
                if (i >= p.r) break;
                PS* h = reinterpret_cast<PS*>(&u[k]);
                const float kf = s_k[i], qf = s_q[i];
#pragma unroll
                for (int e = 0; e < VEC / 2; ++e) {
                    const float2 f = widen(h[e]);
                    const float s0 = rnd_to<TS>(__fadd_rn(f.x, rnd_to<TS>(__fmul_rn(kf, vv[2 * e]))));
                    const float s1 = rnd_to<TS>(__fadd_rn(f.y, rnd_to<TS>(__fmul_rn(kf, vv[2 * e + 1]))));
                    h[e] = Ops<TS>::pack(s0, s1);
                    acc[2 * e] = __fadd_rn(acc[2 * e], __fmul_rn(qf, s0));
                    acc[2 * e + 1] = __fadd_rn(acc[2 * e + 1], __fmul_rn(qf, s1));
                }
                *reinterpret_cast<uint4*>(st + (int64_t)i * p.sr + c) = u[k];
            }
        };
        uint4 ua[U], ub[U];
        load(ua, 0);
        for (int i0 = 0; i0 < p.r; i0 += 2 * U) {
            if (i0 + U < p.r) load(ub, i0 + U);
            update(ua, i0);
            if (i0 + U >= p.r) break;
            if (i0 + 2 * U < p.r) load(ua, i0 + 2 * U);
            update(ub, i0 + U);
        }
        uint4 o;
        PS* oh = reinterpret_cast<PS*>(&o);
#pragma unroll
        for (int e = 0; e < VEC / 2; ++e)
            oh[e] = Ops<TS>::pack(__fdiv_rn(rnd_to<TS>(acc[2 * e]), den), __fdiv_rn(rnd_to<TS>(acc[2 * e + 1]), den));
        *reinterpret_cast<uint4*>(out + c) = o;
    }
}

// ------------------------------------------------------------------ host
size_t align128(size_t x) { return (x + 127) & ~size_t(127); }

// A bf16 [nb, T, width] view (column stride 1) as a 3-D map with 64 x 128 boxes.
int encode_bf16(CUtensorMap* tm, const void* ptr, int64_t width, int64_t T, int64_t nb, int64_t st, int64_t sb,
                const char* what) {
    if (!aligned16(ptr)) return fail(NEED_ERR_UNSUPPORTED, "%s is not 16-byte aligned", what);
    if ((st * 2) % 16 != 0 || (nb > 1 && (sb * 2) % 16 != 0) || st < width || (nb > 1 && sb < st * T))
        return fail(NEED_ERR_UNSUPPORTED, "%s: strides (%lld, %lld) must be 16-byte multiples covering the rows", what,
                    (long long)sb, (long long)st);
    const cuuint64_t dims[3] = {cuuint64_t(width), cuuint64_t(T), cuuint64_t(nb)};
    const cuuint64_t gs[2] = {cuuint64_t(st * 2), cuuint64_t(nb > 1 ? sb * 2 : st * 2 * T)};
    const cuuint32_t box[3] = {64, 128, 1};
    const cuuint32_t es[3] = {1, 1, 1};
    auto fn = encode_fn();
    if (fn == nullptr) return fail(NEED_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    const CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, gs, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(NEED_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled(%s) failed: %d", what, int(r));
    return NEED_OK;
}

#ifndef NEED_ASSOC_PREFIX_COST
#define NEED_ASSOC_PREFIX_COST 0.25  // a state-only tile, in own tiles (two per load, no Q, no outputs)
#endif
#ifndef NEED_ASSOC_SWITCH_COST
#define NEED_ASSOC_SWITCH_COST 1.0  // the first own tile's load after the state-only tiles
#endif
// the chunk-state alternative, in own tiles: its launch, a tile of it, the chunk scan
#ifndef NEED_ASSOC_STATE_LAUNCH_COST
#define NEED_ASSOC_STATE_LAUNCH_COST 3.0
#endif
#ifndef NEED_ASSOC_STATE_TILE_COST
#define NEED_ASSOC_STATE_TILE_COST 0.5
#endif
#ifndef NEED_ASSOC_SCAN_COST
#define NEED_ASSOC_SCAN_COST 1.0
#endif

// Boundaries of at most `nseg` segments over `ntile` tiles that even out the
// CTAs' times when later segments run the tiles before them state-only: a
// segment starting at tile a with n own tiles costs n, plus a * prefix +
// switch when a > 0.  The smallest budget whose greedy cover fits is found by
// bisection; returns the number of segments used and the budget in *cost.
int assoc_segments(int ntile, int nseg, int32_t* seg, double* cost) {
    const double pre = NEED_ASSOC_PREFIX_COST, sw = NEED_ASSOC_SWITCH_COST;
    auto cover = [&](double budget, int32_t* out) {
        int a = 0, s = 0;
        if (out) out[0] = 0;
        while (a < ntile && s < nseg) {
            const double left = budget - (a > 0 ? pre * a + sw : 0.0);
            const int n = std::max(1, static_cast<int>(left + 1e-9));
            a = std::min(ntile, a + n);
            if (out) out[s + 1] = a;
            ++s;
        }
        return a == ntile ? s : -1;
    };
    double lo = 0.0, hi = ntile;  // one segment with every tile fits `hi`
    for (int i = 0; i < 50; ++i) {
        const double mid = 0.5 * (lo + hi);
        (cover(mid, nullptr) > 0 ? hi : lo) = mid;
    }
    *cost = hi;
    return cover(hi, seg);
}

// How a launch splits the sequences into `nseg` segments per sequence (the
// CTAs of all segments fill the SMs once).  Of two plans, the cheaper by the
// cost model above:
//  * two segments, the second re-summing the first's tiles state-only, at
//    boundaries that balance the two;
//  * as many equal segments as the SMs take, after a launch that sums the
//    tiles before the last segment in `nchunk` chunks (`kchunk` per segment)
//    on as many SMs again.
struct AssocPlan {
    int nseg = 1, kchunk = 0, nchunk = 0, recompute = 0;
    int32_t seg[kMaxSeg + 1] = {};
    int32_t chunk[kMaxChunk + 1] = {};
};

int device_sms() {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        cudaGetLastError();
        return 148;
    }
    return sms;
}

AssocPlan assoc_plan(int64_t nb, int64_t T, int64_t d, int sms) {
    AssocPlan pl;
    const int64_t ncb = (d + kCols - 1) / kCols, ntile = (T + kTok - 1) / kTok, per = ncb * nb;
    const int most = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>({ntile, sms / per, kMaxSeg})));
    AssocPlan re;  // at most two segments, no chunk states
    double re_cost = 0.0;
    re.recompute = most > 1;
    re.nseg = assoc_segments(static_cast<int>(ntile), std::min(most, 2), re.seg, &re_cost);
    if (most <= 2) return re;
    pl.nseg = most;
    for (int s = 0; s <= pl.nseg; ++s) pl.seg[s] = static_cast<int32_t>(s * ntile / pl.nseg);
    if (pl.nseg > 1) {
        const int64_t shortest = ntile / pl.nseg;  // >= 1 tile
        pl.kchunk = static_cast<int>(std::max<int64_t>(
            1, std::min<int64_t>({sms / (per * (pl.nseg - 1)), shortest, kMaxChunk / (pl.nseg - 1)})));
        pl.nchunk = (pl.nseg - 1) * pl.kchunk;
        for (int s = 0; s + 1 < pl.nseg; ++s) {
            const int len = pl.seg[s + 1] - pl.seg[s];
            for (int j = 0; j < pl.kchunk; ++j) pl.chunk[s * pl.kchunk + j] = pl.seg[s] + j * len / pl.kchunk;
        }
        pl.chunk[pl.nchunk] = pl.seg[pl.nseg - 1];
    }
    int longest_seg = 0, longest_chunk = 0;
    for (int s = 0; s < pl.nseg; ++s) longest_seg = std::max(longest_seg, pl.seg[s + 1] - pl.seg[s]);
    for (int c = 0; c < pl.nchunk; ++c) longest_chunk = std::max(longest_chunk, pl.chunk[c + 1] - pl.chunk[c]);
    const double cost = NEED_ASSOC_STATE_LAUNCH_COST + NEED_ASSOC_STATE_TILE_COST * longest_chunk +
                        (pl.nchunk > kScanAbove ? NEED_ASSOC_SCAN_COST : 0.0) + longest_seg;
    return cost < re_cost ? pl : re;
}

// workspace: header | q features | k features | masked v | chunk states | chunk z
struct AssocLayout {
    size_t feat, vm, cs, cz, total;
};
AssocLayout assoc_layout(int64_t nb, int64_t T, int64_t d, bool mask, const AssocPlan& pl) {
    AssocLayout l;
    const int64_t ncb = (d + kCols - 1) / kCols;
    l.feat = align128(size_t(nb) * size_t(T) * kRank * 2);
    l.vm = mask ? align128(size_t(nb) * size_t(T) * size_t(d) * 2) : 0;
    l.cs = align128(size_t(pl.nchunk) * size_t(nb) * size_t(ncb) * kCols * kRank * 4);
    l.cz = align128(size_t(pl.nchunk) * size_t(nb) * kRank * 4);
    l.total = WS_HDR_WORDS * 4 + 2 * l.feat + l.vm + l.cs + l.cz;
    return l;
}

AssocPlan plan_for(int64_t nb, int64_t T, int64_t d) {
    return assoc_plan(nb, T, d, T > kTok ? device_sms() : 1);  // one tile: one segment, no device query
}

}  // namespace

extern "C" {

size_t need_assoc_memory_workspace_size(int64_t nb, int64_t T, int64_t d, int32_t has_mask) {
    if (nb < 1 || T < 1 || d < 1 || T > INT32_MAX / 2 || d > INT32_MAX / 2) return WS_HDR_WORDS * 4;
    return assoc_layout(nb, T, d, has_mask != 0, plan_for(nb, T, d)).total;
}

int need_assoc_memory(const need_assoc_args* a, need_stream_t stream) {
    if (a == nullptr) return fail(NEED_ERR_INVALID, "args is null");
    if (a->nb < 1 || a->T < 1 || a->r < 1 || a->d < 1)
        return fail(NEED_ERR_INVALID, "sizes must be >= 1 (nb=%lld T=%lld r=%lld d=%lld)", (long long)a->nb,
                    (long long)a->T, (long long)a->r, (long long)a->d);
    if (a->dtype != NEED_BF16) return fail(NEED_ERR_UNSUPPORTED, "v / out must be bf16 (dtype %d)", a->dtype);
    if (a->qk_dtype != NEED_F32 && a->qk_dtype != NEED_BF16)
        return fail(NEED_ERR_UNSUPPORTED, "q_raw / k_raw must be fp32 or bf16 (dtype %d)", a->qk_dtype);
    if (a->r > kRank) return fail(NEED_ERR_UNSUPPORTED, "r=%lld: at most %d features", (long long)a->r, kRank);
    if (a->d % 8 != 0) return fail(NEED_ERR_UNSUPPORTED, "d=%lld must be a multiple of 8", (long long)a->d);
    if (a->T > INT32_MAX / 2 || a->d > INT32_MAX / 2 || a->nb > 65535 || a->nb * a->T > INT32_MAX / 2)
        return fail(NEED_ERR_UNSUPPORTED, "sizes out of range");
    if (a->q_raw == nullptr || a->k_raw == nullptr || a->v == nullptr || a->out == nullptr)
        return fail(NEED_ERR_INVALID, "q_raw, k_raw, v and out must be non-null");
    const bool mask = a->write_mask != nullptr;
    if (mask && a->mask_dtype != NEED_F32 && a->mask_dtype != NEED_BF16)
        return fail(NEED_ERR_UNSUPPORTED, "write_mask must be fp32 or bf16 (dtype %d)", a->mask_dtype);
    if (a->eps < 0.0) return fail(NEED_ERR_INVALID, "eps must be >= 0");
    if (a->workspace == nullptr || !aligned16(a->workspace))
        return fail(NEED_ERR_WORKSPACE, "workspace is null or not 16-byte aligned");
    const AssocPlan pl = plan_for(a->nb, a->T, a->d);
    const AssocLayout lay = assoc_layout(a->nb, a->T, a->d, mask, pl);
    if (a->workspace_bytes < lay.total)
        return fail(NEED_ERR_WORKSPACE, "workspace has %zu bytes, needs %zu", a->workspace_bytes, lay.total);
    if (!aligned16(a->v)) return fail(NEED_ERR_UNSUPPORTED, "v is not 16-byte aligned");
    if ((a->v_stride_t % 8) != 0 || (a->nb > 1 && (a->v_stride_b % 8) != 0))
        return fail(NEED_ERR_UNSUPPORTED, "v strides must be multiples of 8 elements");

    unsigned char* ws = static_cast<unsigned char*>(a->workspace);
    unsigned char* wp = ws + WS_HDR_WORDS * 4;
    __nv_bfloat16* qf = reinterpret_cast<__nv_bfloat16*>(wp);
    __nv_bfloat16* kf = reinterpret_cast<__nv_bfloat16*>(wp + lay.feat);
    __nv_bfloat16* vm = mask ? reinterpret_cast<__nv_bfloat16*>(wp + 2 * lay.feat) : nullptr;
    float* cs = reinterpret_cast<float*>(wp + 2 * lay.feat + lay.vm);
    float* cz = reinterpret_cast<float*>(wp + 2 * lay.feat + lay.vm + lay.cs);

    FeatArgs f{};
    f.q = a->q_raw;
    f.k = a->k_raw;
    f.qsb = a->q_stride_b;
    f.qst = a->q_stride_t;
    f.ksb = a->k_stride_b;
    f.kst = a->k_stride_t;
    f.qk32 = a->qk_dtype == NEED_F32;
    f.pairs = f.qk32 && a->r % 2 == 0 && (reinterpret_cast<uintptr_t>(a->q_raw) & 7u) == 0 &&
              (reinterpret_cast<uintptr_t>(a->k_raw) & 7u) == 0 && a->q_stride_t % 2 == 0 &&
              a->k_stride_t % 2 == 0 && a->q_stride_b % 2 == 0 && a->k_stride_b % 2 == 0;
    f.mask = a->write_mask;
    f.mask32 = a->mask_dtype == NEED_F32;
    f.msb = a->mask_stride_b;
    f.mst = a->mask_stride_t;
    f.v = static_cast<const __nv_bfloat16*>(a->v);
    f.vsb = a->v_stride_b;
    f.vst = a->v_stride_t;
    f.qf = qf;
    f.kf = kf;
    f.vm = vm;
    f.nb = a->nb;
    f.T = a->T;
    f.r = a->r;
    f.d = a->d;

    if (int rc = ensure_context()) return rc;
    AssocParams P{};
    if (int rc = encode_bf16(&P.tm_q, qf, kRank, a->T, a->nb, kRank, kRank * a->T, "q features")) return rc;
    if (int rc = encode_bf16(&P.tm_k, kf, kRank, a->T, a->nb, kRank, kRank * a->T, "k features")) return rc;
    if (mask) {
        if (int rc = encode_bf16(&P.tm_v, vm, a->d, a->T, a->nb, a->d, a->d * a->T, "masked v")) return rc;
    } else if (int rc = encode_bf16(&P.tm_v, a->v, a->d, a->T, a->nb, a->v_stride_t, a->v_stride_b, "v")) {
        return rc;
    }
    if (int rc = encode_bf16(&P.tm_out, a->out, a->d, a->T, a->nb, a->out_stride_t, a->out_stride_b, "out"))
        return rc;
    P.T = int32_t(a->T);
    P.d = int32_t(a->d);
    P.eps = static_cast<float>(a->eps);
    P.hdr = reinterpret_cast<uint32_t*>(ws);
    P.cs = cs;
    P.cz = cz;
    P.nb = static_cast<int32_t>(a->nb);
    P.ncb = static_cast<int32_t>((a->d + kCols - 1) / kCols);
    P.kchunk = pl.kchunk;
    P.scanned = pl.nchunk > kScanAbove ? 1 : 0;
    P.recompute = pl.recompute;
    std::copy(pl.seg, pl.seg + kMaxSeg + 1, P.seg);
    std::copy(pl.chunk, pl.chunk + kMaxChunk + 1, P.chunk);

    const int64_t rows = a->nb * a->T;
    const int64_t fblocks = (rows + 4 * kFeatRows - 1) / (4 * kFeatRows);
    if (fblocks > INT32_MAX) return fail(NEED_ERR_UNSUPPORTED, "too many tokens");
    assoc_features_kernel<<<static_cast<unsigned>(fblocks), 128, 0, stream>>>(f);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "assoc_features_kernel launch");
    static std::atomic<uint64_t> smem_done{0}, cs_smem_done{0};
    if ((e = ensure_smem(assoc_kernel, SMEM_BYTES, smem_done)) != cudaSuccess)
        return cuda_fail(e, "cudaFuncSetAttribute(assoc_kernel)");
    const dim3 grid(static_cast<unsigned>(P.ncb), static_cast<unsigned>(a->nb), static_cast<unsigned>(pl.nseg));
    if (pl.nchunk > 0) {  // the states entering the later segments
        if ((e = ensure_smem(assoc_state_kernel, CS_SMEM_BYTES, cs_smem_done)) != cudaSuccess)
            return cuda_fail(e, "cudaFuncSetAttribute(assoc_state_kernel)");
        const dim3 cgrid(static_cast<unsigned>(P.ncb), static_cast<unsigned>(a->nb), static_cast<unsigned>(pl.nchunk));
        assoc_state_kernel<<<cgrid, kThreads, CS_SMEM_BYTES, stream>>>(P);
        if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(e, "assoc_state_kernel launch");
        if (P.scanned) {
            const int64_t cs4 = int64_t(a->nb) * P.ncb * kCols * kRank / 4, cz4 = int64_t(a->nb) * kRank / 4;
            const int64_t threads = cs4 + cz4;
            assoc_chunk_scan_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, stream>>>(cs, cz, cs4, cz4,
                                                                                                    pl.nchunk);
            if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(e, "assoc_chunk_scan_kernel launch");
        }
    }
    assoc_kernel<<<grid, kMainThreads, SMEM_BYTES, stream>>>(P);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(e, "assoc_kernel launch");
    return ok();
}

int need_assoc_memory_step(const need_assoc_step_args* a, need_stream_t stream) {
    if (a == nullptr) return fail(NEED_ERR_INVALID, "args is null");
    if (!dtype_ok(a->dtype)) return fail(NEED_ERR_UNSUPPORTED, "dtype %d", a->dtype);
    if (a->qk_dtype != NEED_F32 && a->qk_dtype != NEED_BF16)
        return fail(NEED_ERR_UNSUPPORTED, "q_raw / k_raw must be fp32 or bf16 (dtype %d)", a->qk_dtype);
    if (a->nseq < 1 || a->r < 1 || a->d < 1) return fail(NEED_ERR_INVALID, "sizes must be >= 1");
    if (a->r > kStepMaxRank) return fail(NEED_ERR_UNSUPPORTED, "r=%lld: at most %d features", (long long)a->r, kStepMaxRank);
    const int64_t vec = 16 / dtype_bytes(a->dtype);
    if (a->d % vec != 0 || a->d > INT32_MAX / 2 || a->nseq > INT32_MAX)
        return fail(NEED_ERR_UNSUPPORTED, "d=%lld must be a multiple of %lld", (long long)a->d, (long long)vec);
    if (a->q_raw == nullptr || a->k_raw == nullptr || a->v == nullptr || a->state == nullptr ||
        a->denom == nullptr || a->out == nullptr)
        return fail(NEED_ERR_INVALID, "q_raw, k_raw, v, state, denom and out must be non-null");
    if (a->write_mask != nullptr && a->mask_dtype != NEED_F32 && a->mask_dtype != NEED_BF16)
        return fail(NEED_ERR_UNSUPPORTED, "write_mask must be fp32 or bf16 (dtype %d)", a->mask_dtype);
    if (!aligned16(a->v) || !aligned16(a->state) || !aligned16(a->out) || a->v_stride % vec != 0 ||
        a->out_stride % vec != 0 || a->state_stride_n % vec != 0 || a->state_stride_r % vec != 0)
        return fail(NEED_ERR_UNSUPPORTED, "v, state and out need 16-byte aligned rows");
    if (!(a->eps >= 0.0)) return fail(NEED_ERR_INVALID, "eps must be >= 0");
    StepParams p{a->q_raw, a->k_raw, a->q_stride, a->k_stride, a->qk_dtype == NEED_F32 ? 1 : 0, a->v, a->v_stride,
                 a->write_mask, a->mask_dtype == NEED_F32 ? 1 : 0, a->state, a->state_stride_n, a->state_stride_r,
                 a->denom, a->denom_stride_n, a->slot, a->out, a->out_stride, static_cast<int32_t>(a->r),
                 static_cast<int32_t>(a->d), static_cast<float>(a->eps)};
    const dim3 grid(static_cast<unsigned>(a->nseq));
    if (a->dtype == NEED_BF16) assoc_step_kernel<__nv_bfloat16><<<grid, kStepThreads, 0, stream>>>(p);
    else if (a->dtype == NEED_F16) assoc_step_kernel<__half><<<grid, kStepThreads, 0, stream>>>(p);
    else assoc_step_kernel<float><<<grid, kStepThreads, 0, stream>>>(p);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "assoc_step_kernel launch");
    return ok();
}

}  // extern "C"
