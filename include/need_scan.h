/*
 * need_scan.h -- C ABI of the B200 (sm_100a) recurrent-scan library
 * (need_b200/_lib/libneed_scan.so).
 *
 * The library implements NEED's gated linear recurrence
 *
 *     h[t] = a[t] * h[t-1] + b[t]        (element-wise per channel)
 *
 * and the gate arithmetic its callers wrap around it.  Every entry point takes
 * plain device pointers, element strides and sizes, launches on the given
 * stream, never synchronises and never allocates device memory; scratch comes
 * from a caller-owned workspace (see need_scan_workspace_size).
 *
 * Reference interfaces replaced (NEED, file:line):
 *   need_affine_recurrence_scan  <- need_kernels.affine_recurrence_scan   need_kernels.py:229-264
 *   need_ssd_scan                <- need_kernels.ssd_scan                 need_kernels.py:302-339
 *   need_recurrent_retention_scan<- need_kernels.recurrent_retention_scan need_kernels.py:342-345
 *   need_gated_scan              <- the sigmoid-gated scan its callers compose from
 *                                   torch ops (need_core.py:1630-1638 with a sigmoid decay)
 *   need_ragged_verify           <- the one-token recurrent step applied k times
 *                                   (need_core.py:6410-6431, :1653-1686) for a ragged
 *                                   batch of drafted tokens (generate.py:885-1001)
 *   need_commit_states           <- keeping the state at the accepted prefix
 *                                   (generate.py:1078-1083 appends the accepted tokens)
 *   need_sp_fixup                <- no counterpart (sequence-parallel extension)
 *   need_affine_recurrence_scan_backward <- no counterpart (the reference differentiates
 *                                   its scan with torch autograd, need_kernels.py:177-226)
 *   need_segment_starts          <- no counterpart (resets from the packed stream format
 *                                   of train.py:320-352)
 *   need_ssd_conv_silu           <- the conv + SiLU prologue of StructuredDualRetention
 *                                   (need_core.py:1620-1622), as one kernel
 *   need_assoc_memory            <- HierarchicalMemory._linear_associative_memory
 *                                   (need_core.py:1960-2001), the matrix-state memory
 *   need_assoc_memory_step       <- its one-token step in HierarchicalMemory.stream_step
 *                                   (need_core.py:2067-2080)
 *   need_rms_norm                <- need_kernels.rms_norm (need_kernels.py:266-276; its
 *                                   GPU kernel need_kernels.py:99-107)
 *   need_ssd_scan_rms_norm       <- need_kernels.ssd_scan followed by the block's
 *                                   out_norm (need_core.py:1624-1643), one call
 *
 * Return codes: NEED_OK (0), or a need_status error; need_last_error() gives a
 * message for the calling thread's last failure.  All entry points are
 * reentrant and may be called from several host threads on distinct streams.
 */
#ifndef NEED_SCAN_H
#define NEED_SCAN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NEED_SCAN_ABI_VERSION 2

#if defined(__GNUC__)
#define NEED_API __attribute__((visibility("default")))
#else
#define NEED_API
#endif

typedef struct CUstream_st* need_stream_t; /* == cudaStream_t */

typedef enum {
    NEED_OK = 0,
    NEED_ERR_INVALID = 1,     /* bad argument: null pointer, negative size, bad form */
    NEED_ERR_UNSUPPORTED = 2, /* dtype / alignment / stride the kernels do not take */
    NEED_ERR_CUDA = 3,        /* a CUDA runtime or driver call failed */
    NEED_ERR_WORKSPACE = 4    /* workspace missing or smaller than required */
} need_status;

typedef enum { NEED_F32 = 0, NEED_BF16 = 1, NEED_F16 = 2 } need_dtype;

/* What the streamed inputs in[] hold, and what `out` receives.
 *   NEED_FORM_AFFINE    in[0]=decay a (dtype decay_dtype, or one value per row
 *                       when decay_per_row), in[1]=update b          out = h
 *   NEED_FORM_GATED     in[0]=decay logit z, in[1]=input-gate logit g, in[2]=x
 *                       a = sigmoid(z), b = (1-a)*(sigmoid(g)*x)    out = h
 *   NEED_FORM_SSD       in[0]=dt_raw, in[1]=b_gate, in[2]=u, in[3]=c_gate,
 *                       in[4]=out_gate; a = exp(-(dt_min + dt_scale*sigmoid(dt_raw))),
 *                       b = (1-a)*(sigmoid(b_gate)*u)
 *                       out = (sigmoid(c_gate)*h + d_skip*u) * sigmoid(out_gate)
 *   NEED_FORM_RETENTION in[0]=decay (as AFFINE), in[1]=kv, in[2]=q
 *                       out = q * h
 * Resets: where seg_start[b, t] != 0 the state is zeroed before step t
 * (a[t] := 0; b[t] unchanged).
 *
 * Precision: the state is carried in fp32.  With 16-bit inputs every gate op
 * is rounded to the input dtype at the points where the reference's torch path
 * rounds (need_kernels.py:330-339), and the state is rounded to the input dtype
 * before the SSD / retention epilogue, as the reference's `state_seq` is. */
typedef enum {
    NEED_FORM_AFFINE = 0,
    NEED_FORM_GATED = 1,
    NEED_FORM_SSD = 2,
    NEED_FORM_RETENTION = 3
} need_form;

/* A streamed tensor viewed as [nb, nh, T, C] with channel stride 1.
 * Strides are in elements.  The base must be 16-byte aligned and every stride
 * times the element size a multiple of 16 bytes (dims of size 1 excepted). */
typedef struct {
    const void* ptr;
    int64_t stride_b, stride_h, stride_t;
} need_view;

typedef struct {
    int32_t form;        /* need_form */
    int32_t dtype;       /* need_dtype of in[] other than an AFFINE/RETENTION decay, and of out */
    int32_t decay_dtype; /* AFFINE / RETENTION: need_dtype of in[0] */
    int32_t decay_per_row; /* AFFINE / RETENTION: 1 = in[0] holds one value per (b, h, t),
                              broadcast over C (its view's stride_* index [nb, nh, T]) */
    int64_t nb, nh, T, C;  /* sequence = (b, h); nb * nh independent recurrences of C channels */
    need_view in[5];
    void* out;             /* [nb, nh, T, C], dtype `dtype` */
    int64_t out_stride_b, out_stride_h, out_stride_t;
    const float* d_skip;   /* SSD: [C] fp32 */
    double dt_min, dt_max; /* SSD: dt = dt_min + (dt_max - dt_min) * sigmoid(dt_raw) */
    const float* h0;       /* optional [nb*nh, C] fp32 initial state (contiguous) */
    float* h_final;        /* optional [nb*nh, C] fp32 state after the last token */
    const uint8_t* seg_start; /* optional reset mask indexed [b, t] (shared by the nh heads) */
    int64_t seg_stride_b, seg_stride_t;
    float* summary;        /* optional [nb*nh, C, 2] fp32: (prod of a over T, h_final), the
                              per-slice summary the sequence-parallel combine exchanges */
    float* tile_prod;      /* optional [nb*nh, ceil(T/L), C] fp32: product of a over
                              [0, start of chunk), L = need_scan_chunk_len(form, dtype, ...) */
    float* tile_carry;     /* optional [nb*nh, ceil(T/L), C] fp32: the state entering each chunk */
    void* workspace;       /* >= need_scan_workspace_size(...) bytes, zero-filled before its
                              first use; reusable by later calls on the same stream without
                              clearing; never used by two launches at once */
    size_t workspace_bytes;
    uint32_t* sp_list;     /* sequence parallelism, the slice's list of the tiles its fix-up
                              rewrites, written by need_sp_local_scan and read by need_sp_fixup
                              (GATED); unused (may be null) elsewhere */
    uint64_t sp_list_words; /* its size in 32-bit words, >= need_sp_list_size(...) */
} need_scan_args;

/* Token dtypes of a packed stream (the packer writes uint16 or uint32,
 * train.py:320-335; the dataloader hands int64 windows to the model). */
typedef enum { NEED_TOK_U16 = 0, NEED_TOK_U32 = 1, NEED_TOK_I32 = 2, NEED_TOK_I64 = 3 } need_token_dtype;

/* need_segment_starts: tokens [nb, T] (element strides), reset mask out. */
typedef struct {
    const void* tokens;
    int32_t token_dtype;   /* need_token_dtype */
    int64_t nb, T;
    int64_t tok_stride_b, tok_stride_t;
    int64_t eos_id, bos_id; /* NEED's Special.eos = 2, Special.bos = 1 (need_core.py:50-53) */
    uint8_t* seg_start;    /* out [nb, T]: 1 where a document starts */
    int64_t seg_stride_b, seg_stride_t;
} need_segment_args;

/* need_ssd_conv_silu: the SSD block's input prologue. */
typedef struct {
    int32_t dtype;          /* NEED_BF16 or NEED_F16: u, out, weight and bias */
    int32_t K;              /* taps, 1..4 (NEED's ssd_conv_kernel) */
    int64_t nb, T, C;       /* C a multiple of 8 */
    const void* u;          /* [nb, T, C], channel stride 1, 16-byte aligned rows */
    int64_t u_stride_b, u_stride_t;
    void* out;              /* [nb, T, C], same layout rules */
    int64_t out_stride_b, out_stride_t;
    const void* weight;     /* [C, K] taps, oldest first: nn.Conv1d(C, C, K, groups=C).weight[:, 0, :] */
    int64_t w_stride_c, w_stride_k;
    const void* bias;       /* [C] or null */
    const uint8_t* seg_start; /* optional reset mask [nb, T]: the window stops at a segment start */
    int64_t seg_stride_b, seg_stride_t;
} need_conv_args;

/* need_ssd_conv_scan: the SSD block's depthwise conv, applied inside the scan. */
typedef struct {
    int32_t K;              /* taps, 1..4 (NEED's ssd_conv_kernel) */
    const void* weight;     /* [C, K] taps, oldest first, the stream dtype (as need_conv_args.weight) */
    int64_t w_stride_c, w_stride_k;
    const void* bias;       /* [C] or null, the stream dtype */
} need_ssd_conv;

/* need_rms_norm: RMSNorm over the C channels of nb x T rows. */
typedef struct {
    int32_t dtype;          /* x and out: NEED_BF16, NEED_F16 or NEED_F32 */
    int32_t weight_dtype;   /* NEED_F32 or `dtype` */
    int64_t nb, T, C;       /* C a multiple of 16 bytes' worth of elements */
    const void* x;          /* [nb, T, C], channel stride 1, 16-byte aligned rows */
    int64_t x_stride_b, x_stride_t;
    void* out;              /* [nb, T, C], same rules; may be x (in place) */
    int64_t out_stride_b, out_stride_t;
    const void* weight;     /* [C], 16-byte aligned */
    double eps;
} need_norm_args;

/* need_assoc_memory: the matrix-state associative memory of HierarchicalMemory. */
typedef struct {
    int32_t dtype;          /* v and out: NEED_BF16 */
    int32_t qk_dtype;       /* q_raw and k_raw: NEED_F32 (the model's fp32 projections) or NEED_BF16 */
    int64_t nb, T, r, d;    /* r <= 64 features; d a multiple of 8 */
    const void* q_raw;      /* [nb, T, r], feature stride 1 */
    int64_t q_stride_b, q_stride_t;
    const void* k_raw;      /* [nb, T, r], feature stride 1 */
    int64_t k_stride_b, k_stride_t;
    const void* v;          /* [nb, T, d], column stride 1, 16-byte aligned rows */
    int64_t v_stride_b, v_stride_t;
    const void* write_mask; /* optional [nb, T]: write weights, rounded to bf16 and clamped to [0, 1] */
    int32_t mask_dtype;     /* NEED_F32 or NEED_BF16 */
    int64_t mask_stride_b, mask_stride_t;
    void* out;              /* [nb, T, d], column stride 1, 16-byte aligned rows */
    int64_t out_stride_b, out_stride_t;
    double eps;             /* denominator floor (the reference's 1e-6) */
    void* workspace;        /* >= need_assoc_memory_workspace_size(...) bytes, 16-byte aligned; the
                               first 128 bytes zero-filled before first use (the error word) */
    size_t workspace_bytes;
} need_assoc_args;

/* need_assoc_memory_step: one token of the associative memory per sequence,
 * against per-sequence states kept between calls (decode). */
typedef struct {
    int32_t dtype;          /* v, out, state and denom: the model dtype (NEED_BF16, NEED_F16, NEED_F32) */
    int32_t qk_dtype;       /* q_raw and k_raw: NEED_F32 or NEED_BF16 */
    int64_t nseq, r, d;     /* r <= 256; d a multiple of 16 bytes' worth of elements */
    const void* q_raw;      /* [nseq, r], feature stride 1 */
    int64_t q_stride;
    const void* k_raw;      /* [nseq, r], feature stride 1 */
    int64_t k_stride;
    const void* v;          /* [nseq, d], 16-byte aligned rows */
    int64_t v_stride;
    const void* write_mask; /* optional [nseq] contiguous, rounded to the model dtype and clamped to [0, 1] */
    int32_t mask_dtype;     /* NEED_F32 or NEED_BF16 */
    void* state;            /* [nslots, r, d], column stride 1, 16-byte aligned rows; updated in place */
    int64_t state_stride_n, state_stride_r;
    void* denom;            /* [nslots, r], feature stride 1; updated in place */
    int64_t denom_stride_n;
    const int32_t* slot;    /* optional [nseq]: state row of sequence i (default i) */
    void* out;              /* [nseq, d], 16-byte aligned rows */
    int64_t out_stride;
    double eps;             /* denominator floor (the reference's 1e-6) */
} need_assoc_step_args;

/* Version of this header the library was built from. */
NEED_API int need_abi_version(void);

/* Message for the calling thread's most recent failure ("" if none). */
NEED_API const char* need_last_error(void);

/* Tokens per tile along T for a call (the chunk length tile_prod is indexed by). */
NEED_API int64_t need_scan_chunk_len(int32_t form, int32_t dtype, int32_t decay_dtype, int32_t decay_per_row);

/* Workspace bytes a call with these sizes needs. */
NEED_API size_t need_scan_workspace_size(int32_t form, int32_t dtype, int32_t decay_dtype,
                                int32_t decay_per_row, int64_t nb, int64_t nh, int64_t T,
                                int64_t C);

/* Reads (and clears) the workspace's device-side error word: bit 0 = a look-back
 * wait gave up, bit 1 = a tile load (or tensor-core) wait gave up, bit 2 = a
 * sequence-parallel fix-up found a tile id outside the slice in sp_list (its
 * local scan did not run as a rank > 0) and skipped it.
 * Synchronises `stream`. */
NEED_API int need_workspace_error(void* workspace, uint32_t* error_out, need_stream_t stream);

/* Test hook, no counterpart in the reference: the number of look-back polls
 * after which a scan's wait for a predecessor tile gives up (sets bit 0 of the
 * workspace error word, takes a zero carry and lets the launch finish), for
 * every scan launched afterwards in this process; 0 restores the default
 * (2^22 polls, a few seconds).  Lets a test make a wait run out quickly
 * without a fault. */
NEED_API void need_test_set_lookback_polls(uint32_t polls);

/* need_kernels.affine_recurrence_scan (need_kernels.py:229-264): args->form must be
 * NEED_FORM_AFFINE. */
NEED_API int need_affine_recurrence_scan(const need_scan_args* args, need_stream_t stream);

/* The backward of need_affine_recurrence_scan: no counterpart in the reference,
 * whose gradient is torch autograd through the chunked CPU scan
 * (need_kernels.py:177-226) or through torch's associative_scan on CUDA
 * (need_kernels.py:245-262).  For h_t = a_t h_{t-1} + b_t and the output
 * gradient g it writes the adjoint
 *     lam_t = g_t + a_{t+1} lam_{t+1}   (lam_{T-1} = g_{T-1}),
 * which is the gradient of b; the gradient of a is lam_t * h_{t-1}.
 * args->form = NEED_FORM_AFFINE; in[0] is the forward's decay (per channel or
 * per row, as for the forward), in[1] is g, out receives lam (dtype `dtype`),
 * h_final optionally receives lam_0 in fp32 (the gradient of an initial state
 * is a_0 lam_0).  seg_start, h0, summary and the tile records must be null;
 * T >= 2.  Workspace as for the forward. */
NEED_API int need_affine_recurrence_scan_backward(const need_scan_args* args, need_stream_t stream);

/* The reset mask of packed windows, derived on the GPU: no counterpart in the
 * reference (its scan has no resets; its packer, train.py:320-352, separates
 * documents with EOS after each and one BOS at the start of the stream).
 * seg_start[b, t] = 1 at t = 0, after an EOS (tokens[b, t-1] == eos_id) and at
 * a BOS (tokens[b, t] == bos_id); 0 elsewhere. */
NEED_API int need_segment_starts(const need_segment_args* args, need_stream_t stream);

/* u = silu(causal depthwise conv_K(u_raw)), the SSD block's prologue
 * (need_core.py:1620-1622: nn.Conv1d with padding K-1 trimmed to T, then
 * F.silu), fused into one pass; no counterpart as a single call in the
 * reference.  The conv is accumulated in fp32 and rounded to `dtype`, SiLU is
 * computed in fp32 and rounded again (the reference's rounding points).  With
 * seg_start, inputs before a token's segment start count as 0. */
NEED_API int need_ssd_conv_silu(const need_conv_args* args, need_stream_t stream);

/* need_kernels.ssd_scan (need_kernels.py:302-339): args->form == NEED_FORM_SSD. */
NEED_API int need_ssd_scan(const need_scan_args* args, need_stream_t stream);

/* need_kernels.rms_norm on the GPU (need_kernels.py:266-276), with the
 * arithmetic of the reference's GPU kernel (need_kernels.py:99-107): per row,
 * x in fp32, inv = rsqrt(sum(x^2) / C + eps), out = (x * inv) * weight as two
 * fp32 products, rounded once to `dtype`.  The row's sum is added in a fixed
 * order, so repeated calls give identical results. */
NEED_API int need_rms_norm(const need_norm_args* args, need_stream_t stream);

/* need_ssd_scan followed by StructuredDualRetention's out_norm
 * (need_core.py:1624-1643: out_norm(ssd_scan(...)), an RMSNorm over the C
 * channels of each token) in one call: the scan writes `out`, then
 * need_rms_norm normalises `out` in place while it is still in L2.  `out`
 * receives, per token, y * rsqrt(sum_c(y^2) / C + eps) * weight, where y is
 * need_ssd_scan's output in `dtype` (need_rms_norm's arithmetic).  weight is
 * [C], NEED_F32 or `dtype` (weight_dtype), 16-byte aligned; nh must be 1.
 * Workspace as for need_ssd_scan. */
NEED_API int need_ssd_scan_rms_norm(const need_scan_args* args, const void* norm_weight, int32_t weight_dtype,
                                    double eps, need_stream_t stream);

/* need_ssd_scan with the block's input prologue folded in
 * (need_core.py:1620-1629: u = F.silu(dwconv(u)[..., :T]), then ssd_scan):
 * in[2] holds the RAW u (in_proj's u chunk).  Each tile applies the causal
 * depthwise conv + SiLU to its rows as they land, with need_ssd_conv_silu's
 * arithmetic and resets bit for bit, and the scan and its D*u epilogue use the
 * result, so `out` equals need_ssd_conv_silu followed by need_ssd_scan without
 * the intermediate round trip through HBM.  With norm_weight (non-null) the
 * block's out_norm follows as in need_ssd_scan_rms_norm.  16-bit dtypes; nh == 1.
 * Replaces need_core.py's dwconv + F.silu + need_kernels.ssd_scan sequence. */
NEED_API int need_ssd_conv_scan(const need_scan_args* args, const need_ssd_conv* conv, const void* norm_weight,
                                int32_t weight_dtype, double eps, need_stream_t stream);

/* need_kernels.recurrent_retention_scan (need_kernels.py:342-345):
 * args->form == NEED_FORM_RETENTION. */
NEED_API int need_recurrent_retention_scan(const need_scan_args* args, need_stream_t stream);

/* The sigmoid-gated scan (need_core.py:1630-1638 with decay = sigmoid(z)):
 * args->form == NEED_FORM_GATED. */
NEED_API int need_gated_scan(const need_scan_args* args, need_stream_t stream);

/* Bytes of the static scratch array behind need_gated_scan_noalloc: a 128-byte
 * header plus 8 MiB of look-back records, 32 bytes per channel of each tile
 * (2048 tiles of 128 channels, or 1024 of 256). */
#define NEED_GATED_SCAN_NOALLOC_SCRATCH_BYTES (128 + 1024 * 8192)

/* need_gated_scan for callers that cannot allocate device memory where they run
 * the scan -- e.g. an inference-engine plugin whose enqueue step may not
 * allocate, a serving loop that cannot afford cudaMalloc's implicit
 * device-wide synchronisation, or a runtime that owns a fixed memory budget.
 * No counterpart in the reference.
 *
 * It takes args->workspace / workspace_bytes as unused and instead uses a
 * static device array of NEED_GATED_SCAN_NOALLOC_SCRATCH_BYTES bytes, which
 * every GPU that loads this library holds until the process exits.  A call
 * whose scan needs more scratch than that (more tiles than the array has
 * records for; need_scan_workspace_size gives the bytes a scan needs) fails
 * with NEED_ERR_WORKSPACE and launches nothing.  The first call on each device
 * looks up the array's device address (cudaGetSymbolAddress) and zero-fills the
 * array with cudaMemsetAsync on `stream`, ordered before that call's launch;
 * make that first call before any stream capture.  The address is kept for the
 * life of the process, so after cudaDeviceReset neither this entry point nor
 * need_gated_scan_noalloc_error may be called again.  Each call clears the
 * array's error word on `stream` (so that a wait that gave up in an earlier
 * call does not cut this call's waits short) and launches the same kernel as
 * need_gated_scan, with the same results bit for bit.  All calls share the one
 * array: calls that overlap on the GPU (different streams or host threads at
 * once) race on it; calls that run one after another, on any stream, are fine.
 * It allocates nothing (no cudaMalloc or cudaFree). */
NEED_API int need_gated_scan_noalloc(const need_scan_args* args, need_stream_t stream);

/* Reads and clears the error word of need_gated_scan_noalloc's static array:
 * bit 0 = a look-back wait gave up, bit 1 = a tile load wait gave up, as for
 * need_workspace_error; after either the call's outputs are not valid.  Synchronises `stream`.
 * Call it after a need_gated_scan_noalloc call and before the next one (the
 * next call clears the word).  Like need_workspace_error for a caller's
 * workspace.  No counterpart in the reference. */
NEED_API int need_gated_scan_noalloc_error(uint32_t* error_out, need_stream_t stream);

/* Workspace bytes need_assoc_memory needs: a 128-byte header, the bf16
 * feature-mapped q and k ([nb, T, 64] each), with a write mask the masked
 * values [nb, T, d], and when the sequences are cut into more than two
 * segments the fp32 chunk states that start the later segments (at most one
 * 32 KB state per SM).  The split follows the current device's SM count: ask
 * on the device that runs the call. */
NEED_API size_t need_assoc_memory_workspace_size(int64_t nb, int64_t T, int64_t d, int32_t has_mask);

/* HierarchicalMemory._linear_associative_memory (need_core.py:1960-2001):
 * with q = elu(q_raw) + 1 and k = elu(k_raw) + 1 rounded to bf16 (and k, v
 * scaled by the write mask, each product rounded to bf16, need_core.py:1977-1984),
 *     out[b, t] = (sum_{s<=t} (q_t . k_s) v_s) / max(sum_{s<=t} q_t . k_s, eps),
 * rounded once to bf16.  The reference evaluates the same sums in chunks of
 * memory_chunk_size tokens with its running state and every partial product
 * rounded to the model dtype; here the products are bf16 tensor-core operands
 * (the intra-tile scores q_t . k_s and the state rounded to bf16 for the
 * second product) with fp32 accumulation, and the denominator is fp32.  The
 * chunk length therefore does not enter. */
NEED_API int need_assoc_memory(const need_assoc_args* args, need_stream_t stream);

/* HierarchicalMemory.stream_step's associative memory for one token of each
 * sequence (need_core.py:2067-2080), with the reference's model-dtype
 * arithmetic: q = elu(q_raw) + 1 and k = elu(k_raw) + 1 rounded to the model
 * dtype (k and v scaled by the write mask, rounded); then, each op rounded to
 * the model dtype,
 *     state += k (x) v,   denom += k,
 *     out = (q . state) / max(sum_i q_i denom_i, eps),
 * where q . state and the sum are fp32 sums over the features in feature
 * order.  state and denom are read and written in place (one sequence per
 * row, or per slot[i]); sequences must not share a slot within one call. */
NEED_API int need_assoc_memory_step(const need_assoc_step_args* args, need_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Ragged decode / speculative verify                                        */
/* ------------------------------------------------------------------------ */

typedef struct {
    int32_t form;          /* NEED_FORM_GATED, NEED_FORM_SSD or NEED_FORM_RETENTION */
    int32_t dtype;         /* NEED_BF16, NEED_F16 or NEED_F32: states, inputs and outputs */
    int64_t nseq, C;
    void* states;          /* [nslots, C] state pool, read only here */
    const int32_t* slot;   /* optional [nseq]: pool row of sequence i (default i) */
    const int32_t* cu_k;   /* [nseq + 1] offsets of each sequence's drafted tokens */
    int64_t total_k;       /* cu_k[nseq] (rows of the packed inputs) */
    const void* in[5];     /* packed [total_k, C] contiguous: GATED z, g, x;
                              SSD dt_raw, b_gate, u, c_gate, out_gate;
                              RETENTION in[0] = decay [total_k, C / head_dim] (one value
                              per head), in[1..3] = k, v, q */
    const float* d_skip;   /* SSD: [C] fp32 */
    double dt_min, dt_max;
    void* y;               /* [total_k, C] output of each drafted token */
    void* states_k;        /* [total_k, C] state after each drafted token */
    int64_t head_dim;      /* RETENTION: channels per head (a multiple of 8 dividing C) */
    /* SSD only, optional: the block's causal depthwise conv (need_core.py:6395-6414).
     * With conv_k in 2..4, in[2] holds the raw u, and every drafted token first
     * takes the conv step from its sequence's history and SiLU, in the model
     * dtype: full = [hist, u]; u_conv = sum_j (full_j * w[c, j]) (each product
     * rounded, the sum in fp32 in tap order, rounded) + bias (rounded);
     * hist := full[1:]; u_act = silu(u_conv) (fp32, rounded).  conv_k = 0: in[2]
     * is u_act and the conv fields are unused. */
    int32_t conv_k;
    const void* conv_weight; /* [C, conv_k] contiguous, in `dtype` (the fp32 weight cast as
                                the reference casts it) */
    const void* conv_bias;   /* optional [C] in `dtype` */
    const void* conv_hist;   /* [nslots, C, conv_k - 1] in `dtype`: the raw u of each pool
                                row's last conv_k - 1 tokens, oldest first (the reference's
                                ssd_conv_hist); read only here */
    void* conv_hist_k;       /* [total_k, C, conv_k - 1]: the history after each drafted
                                token; commit it with need_commit_states over rows of
                                C * (conv_k - 1) elements */
} need_verify_args;

/* k_i one-token steps per sequence from its pooled state, in the model dtype's
 * arithmetic (need_core.py:6420-6428; RETENTION: SelectiveRetention's step
 * state = decay * state + k * v, y = q * state, need_core.py:1590-1592).  The
 * pool is not modified. */
NEED_API int need_ragged_verify(const need_verify_args* args, need_stream_t stream);

/* states[slot[i]] := states_k[cu_k[i] + accept_len[i] - 1] when accept_len[i] > 0;
 * accept_len[i] must lie in [0, cu_k[i+1] - cu_k[i]] (clamped on device).  Rows
 * are C elements; the SSD conv history commits with the same call over rows of
 * C * (conv_k - 1) elements (conv_hist, conv_hist_k). */
NEED_API int need_commit_states(int32_t dtype, int64_t nseq, int64_t C, void* states,
                       const int32_t* slot, const void* states_k, const int32_t* cu_k,
                       const int32_t* accept_len, need_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Sequence parallelism (T sharded over ranks)                               */
/* ------------------------------------------------------------------------ */

/* Step 1 of the sequence-parallel gated scan on rank `rank`: the scan of this
 * rank's T-slice from a zero state (form GATED; `summary`, `tile_prod` and
 * `tile_carry` required), as need_gated_scan.  For rank > 0 the tiles that
 * need_sp_fixup will rewrite -- those whose product of a before them exceeds
 * 2^-24 on some channel -- are scanned for their maps, listed in
 * args->sp_list, and their output rows receive the tile's rounded updates
 * b = (1 - a) * (sigmoid(g) * x) instead of outputs (the fix-up re-scans from
 * them): call need_sp_fixup with the same args before reading `out`.
 * Replaces no reference interface (the reference has no distributed scan). */
NEED_API int need_sp_local_scan(const need_scan_args* args, int32_t rank, need_stream_t stream);

/* Words of need_scan_args.sp_list for a GATED slice of this shape: a count
 * (4 words) and one tile id per tile; 0 for an unknown dtype. */
NEED_API size_t need_sp_list_size(int32_t dtype, int64_t nb, int64_t nh, int64_t T, int64_t C);

/* After a rank scanned its T-slice from a zero state (with `summary`,
 * `tile_prod` and `tile_carry` requested) and gathered every rank's summary
 * into `all_summary` [nranks, nb*nh, C, 2], this applies the carry from ranks
 * < rank: carry = compose(summary[0..rank-1]); the affected tiles are
 * re-scanned from the corrected fp32 state tile_carry + tile_prod * carry, with
 * the scan's own arithmetic, and their outputs rewritten; later tiles are left
 * as they are (their correction is below fp32 resolution of the carry).
 * GATED: the tiles need_sp_local_scan listed in args->sp_list (tile_prod
 * above 2^-24 on some channel), in one launch, from their decay logits in[0]
 * and the updates b the local scan left in `out`.  AFFINE: every tile whose
 * correction is non-zero on some channel.  It also corrects h_final / summary
 * when given. */
NEED_API int need_sp_fixup(const need_scan_args* args, const float* all_summary, int32_t nranks,
                  int32_t rank, need_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* NEED_SCAN_H */
