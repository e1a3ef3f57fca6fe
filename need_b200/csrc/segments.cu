// segments.cu -- packed-segment starts from a packed token stream, on the GPU.
//
// NEED packs a corpus as one flat stream: BOS once, then every document
// followed by EOS (train.py:320-352, pack_text_tokens_to_bin with
// add_eos=True); the dataloader cuts [B, T] windows out of it
// (train.py:406-418).  A window's state must restart where a document
// starts: at t = 0, right after an EOS, and at a BOS.  This kernel writes that
// reset mask, seg_start[b, t] in {0, 1}, which every scan entry point takes.
//
// HBM-bound and tiny (a [16, 4096] int64 window is 0.5 MB): one thread per 16
// consecutive tokens of a row, one 16-byte store of flags when the mask rows
// are contiguous and aligned.
#include <cuda_runtime.h>
#include <stdint.h>

#include "host_common.h"
#include "need_scan.h"

using namespace need;

namespace {

struct SegParams {
    const void* tok;
    int64_t sb, st;
    int64_t nb, T;
    int64_t eos, bos;
    uint8_t* seg;
    int64_t gb, gt;
};

template <typename TI>
__global__ void __launch_bounds__(256) segment_kernel(const SegParams p) {
    const int64_t chunks = (p.T + 15) / 16;
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= p.nb * chunks) return;
    const int64_t b = i / chunks, t0 = (i - b * chunks) * 16;
    const TI* row = static_cast<const TI*>(p.tok) + b * p.sb;
    int64_t prev = t0 > 0 ? static_cast<int64_t>(row[(t0 - 1) * p.st]) : -1;
    uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int64_t t = t0 + j;
        if (t < p.T) {
            const int64_t cur = static_cast<int64_t>(row[t * p.st]);
            const uint32_t start = (t == 0 || prev == p.eos || cur == p.bos) ? 1u : 0u;
            w[j >> 2] |= start << (8 * (j & 3));
            prev = cur;
        }
    }
    uint8_t* out = p.seg + b * p.gb + t0 * p.gt;
    if (p.gt == 1 && t0 + 16 <= p.T && (reinterpret_cast<uintptr_t>(out) & 15u) == 0) {
        *reinterpret_cast<uint4*>(out) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
        for (int j = 0; j < 16 && t0 + j < p.T; ++j) out[j * p.gt] = static_cast<uint8_t>((w[j >> 2] >> (8 * (j & 3))) & 1u);
    }
}

}  // namespace

extern "C" int need_segment_starts(const need_segment_args* a, need_stream_t stream) {
    if (a == nullptr || a->tokens == nullptr || a->seg_start == nullptr) return fail(NEED_ERR_INVALID, "null argument");
    if (a->nb < 1 || a->T < 1) return fail(NEED_ERR_INVALID, "sizes must be >= 1 (nb=%lld T=%lld)", (long long)a->nb,
                                            (long long)a->T);
    SegParams p{a->tokens, a->tok_stride_b, a->tok_stride_t, a->nb, a->T, a->eos_id, a->bos_id,
                a->seg_start, a->seg_stride_b, a->seg_stride_t};
    const int64_t threads = a->nb * ((a->T + 15) / 16);
    const unsigned blocks = static_cast<unsigned>((threads + 255) / 256);
    switch (a->token_dtype) {
        case NEED_TOK_U16: segment_kernel<uint16_t><<<blocks, 256, 0, stream>>>(p); break;
        case NEED_TOK_U32: segment_kernel<uint32_t><<<blocks, 256, 0, stream>>>(p); break;
        case NEED_TOK_I32: segment_kernel<int32_t><<<blocks, 256, 0, stream>>>(p); break;
        case NEED_TOK_I64: segment_kernel<int64_t><<<blocks, 256, 0, stream>>>(p); break;
        default: return fail(NEED_ERR_UNSUPPORTED, "token dtype %d", a->token_dtype);
    }
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ok() : cuda_fail(e, "segment_kernel launch");
}
