/*
 * semicrf.h -- C ABI of the B200 (sm_100a) streaming semi-CRF scan.
 *
 * This is the drop-in boundary for the hot path of torch-semimarkov 0.2.0
 * (src/torch_semimarkov/streaming/).  The reference binds that path from
 * Python through Triton launchers; each entry point below replaces one of
 * them (file:line in the reference project):
 *
 *   semicrf_forward            launch_streaming_triton_kernel
 *                              (streaming/triton_forward.py:554-714) and the
 *                              forward of SemiCRFStreamingTriton
 *                              (streaming/autograd.py:187-226)
 *   semicrf_backward           launch_streaming_triton_backward
 *                              (streaming/triton_backward.py:556-790) and the
 *                              backward of SemiCRFStreamingTriton
 *                              (streaming/autograd.py:228-267)
 *   semicrf_viterbi            SemiMarkovCRFHead.decode_with_traceback /
 *                              _traceback_single (nn.py:360-531)
 *   semicrf_score_gold         score_gold_vectorized (helpers.py:365-544)
 *   semicrf_score_gold_backward  autograd of score_gold_vectorized
 *   semicrf_checkpoint_interval  _compute_checkpoint_interval
 *                              (streaming/pytorch_reference.py:25-45)
 *   semicrf_edge_scan_forward  the edge-tensor scan: launch_triton_kernel
 *                              (triton_scan.py:594-656) and the forward of
 *                              SemiCRFTritonForward (triton_scan.py:738-752)
 *   semicrf_edge_scan_backward the backward of SemiCRFTritonForward
 *                              (triton_scan.py:754-770)
 *
 * Conventions
 *  - All tensors are device pointers to contiguous row-major float32 (int64
 *    for lengths/labels) on the current CUDA device.
 *  - The caller owns every buffer.  The library never allocates or frees
 *    device memory: scratch space is passed in, sized by the matching
 *    *_workspace_size query.
 *  - `stream` is a cudaStream_t (NULL = legacy default stream).  Calls only
 *    enqueue work; they do not synchronise.
 *  - Return value: SEMICRF_OK or an error code; semicrf_strerror() names it.
 */
#ifndef SEMICRF_H_
#define SEMICRF_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SEMICRF_ABI_VERSION 1

enum semicrf_status {
    SEMICRF_OK = 0,
    SEMICRF_ERR_INVALID_ARGUMENT = 1, /* bad sizes / null pointers / K < 1 */
    SEMICRF_ERR_UNSUPPORTED = 2,      /* shape outside the supported range */
    SEMICRF_ERR_WORKSPACE = 3,        /* workspace smaller than queried */
    SEMICRF_ERR_CUDA = 4,             /* a CUDA launch failed */
    SEMICRF_ERR_SEMIRING = 5          /* semiring is neither log nor max */
};

enum semicrf_semiring { SEMICRF_LOG = 0, SEMICRF_MAX = 1 };

/* One streaming problem: the arguments of semi_crf_streaming_forward
 * (streaming/autograd.py:270-281). */
typedef struct semicrf_problem {
    int64_t batch;                /* B */
    int64_t T;                    /* cum_scores has T+1 rows */
    int64_t K;                    /* max duration; durations 1..max(1,K-1) */
    int64_t C;                    /* number of labels */
    const float* cum_scores;      /* (B, T+1, C) */
    const float* transition;      /* (C, C) [src, dst] or (K, C, C) */
    int32_t transition_ndim;      /* 2 or 3 */
    int32_t semiring;             /* enum semicrf_semiring */
    const float* duration_bias;   /* (K, C) */
    const int64_t* lengths;       /* (B,), each in [0, T] */
    const float* proj_start;      /* (B, T, C) or NULL */
    const float* proj_end;        /* (B, T, C) or NULL */
    int64_t checkpoint_interval;  /* S >= K (see semicrf_checkpoint_interval) */
    int32_t backward_mode;        /* what the forward keeps for the backward:
                                     SEMICRF_KEEP_ALPHA: float64 alpha tables,
                                       O(B*T*C) memory, no recompute;
                                     SEMICRF_RECOMPUTE: ring checkpoints every
                                       S' >= S, O(B*T/S*K*C) memory, alpha is
                                       recomputed segment-parallel */
    int32_t chunk_warmup;         /* time chunking of the log-semiring chains
                                     when the forward keeps SEMICRF_KEEP_ALPHA
                                     state: 0 = automatic (when the batch
                                     leaves SMs idle), -1 = never, > 0 = force
                                     it with (bits 0..15) this many warm-up
                                     positions and (bits 16..30, 0 = none) a
                                     second, longer warm-up.  Chunks start
                                     early from a guessed state and are
                                     accepted only where their state matches
                                     the previous chunk's to 1e-10 in
                                     projective distance; other sequences
                                     rerun their chunks with the second
                                     warm-up, and those that still do not
                                     join are recomputed as one chain. */
} semicrf_problem;

enum semicrf_backward_mode { SEMICRF_KEEP_ALPHA = 0, SEMICRF_RECOMPUTE = 1 };

/* _compute_checkpoint_interval: max(K, floor(sqrt(T*K))). */
int64_t semicrf_checkpoint_interval(int64_t T, int64_t K);

/* Bytes of state semicrf_forward keeps for semicrf_backward: the float64
 * log partition (B,) first, then the chain tables (SEMICRF_KEEP_ALPHA) or the
 * normalised restart records (SEMICRF_RECOMPUTE). */
size_t semicrf_saved_size(const semicrf_problem* p);
size_t semicrf_forward_workspace_size(const semicrf_problem* p);

/* Forward scan.  Writes partition (B,) and, when ring_checkpoints is not
 * NULL, the ring buffer of alpha at every multiple of S in the reference
 * layout (B, num_ring_checkpoints, K, C) (NEG_INF = -1e9 where unset;
 * checkpoint 0 holds alpha[0] = 0 in slot 0).  When saved is not NULL the
 * state needed by semicrf_backward is written there; in the log semiring with
 * SEMICRF_KEEP_ALPHA the ring checkpoints are then read off the kept alpha
 * tables after the chains have run. */
int semicrf_forward(const semicrf_problem* p, float* partition, float* ring_checkpoints,
                    int64_t num_ring_checkpoints, void* saved, void* workspace,
                    size_t workspace_bytes, void* stream);

size_t semicrf_backward_workspace_size(const semicrf_problem* p);

/* Backward: gradients of sum_b grad_output[b] * partition[b].
 * grad_cum (B,T+1,C), grad_transition (C,C) or (K,C,C), grad_duration_bias
 * (K,C) are always written; grad_proj_start / grad_proj_end (B,T,C) when the
 * corresponding projection is present.  `saved` is the buffer filled by
 * semicrf_forward for the same problem. */
int semicrf_backward(const semicrf_problem* p, const void* saved, const float* grad_output,
                     float* grad_cum, float* grad_transition, float* grad_duration_bias,
                     float* grad_proj_start, float* grad_proj_end, void* workspace,
                     size_t workspace_bytes, void* stream);

size_t semicrf_viterbi_workspace_size(const semicrf_problem* p);

/* Max-semiring scan with compact (k, c_src) backpointers and a GPU
 * backtrace.  scores (B,); segments of sequence b are written at offset b*T
 * of seg_start/seg_end/seg_label/seg_score, in order, nseg[b] of them.
 * Sequences with length 0 or longer than max_traceback_length get nseg = 0
 * (their score is still written).  seg_score follows nn.py:533-555. */
int semicrf_viterbi(const semicrf_problem* p, int64_t max_traceback_length, float* scores,
                    int32_t* seg_start, int32_t* seg_end, int32_t* seg_label,
                    double* seg_score, int32_t* nseg, void* workspace, size_t workspace_bytes,
                    void* stream);

/* Gold-segmentation score (helpers.py:365-544): out (B,). transition (C,C). */
int semicrf_score_gold(int64_t B, int64_t T, int64_t K, int64_t C, const float* cum_scores,
                       const int64_t* labels, const int64_t* lengths, const float* transition,
                       const float* duration_bias, float* out, void* stream);

/* Its gradient: grad_cum (B,T+1,C) is overwritten; grad_transition (C,C)
 * and grad_duration_bias (K,C) are overwritten with sum_b grad_out[b]*d/d. */
int semicrf_score_gold_backward(int64_t B, int64_t T, int64_t K, int64_t C,
                                const int64_t* labels, const int64_t* lengths,
                                const float* grad_out, float* grad_cum, float* grad_transition,
                                float* grad_duration_bias, void* workspace,
                                size_t workspace_bytes, void* stream);
size_t semicrf_score_gold_workspace_size(int64_t B, int64_t T, int64_t K, int64_t C);

/* Edge-tensor scan (triton_scan.py:163-273, semi_crf_triton_forward at
 * :773-860): log potentials edge (B, N-1, K, C, C), indexed [b][start]
 * [duration index][new label][previous label], for sequences of N
 * positions.  partition (B) = (+)_c beta[L-1, c] with beta[0] = 0 and
 * beta[n, c] = (+)_{k, c'} (beta[n-k, c'] + edge[n-k, min(k, K-1), c, c']),
 * k = 1 .. max(1, min(K-1, n)); (+) = logsumexp (SEMICRF_LOG) or max.
 * Lengths 0 or above N give -1e9, length 1 gives (+) over zeros.  `saved`
 * (may be NULL when no backward follows) keeps what the backward needs;
 * edge may be NULL when N == 1. */
size_t semicrf_edge_scan_saved_size(int64_t B, int64_t N, int64_t K, int64_t C, int semiring);
int semicrf_edge_scan_forward(int64_t B, int64_t N, int64_t K, int64_t C, const float* edge,
                              const int64_t* lengths, int semiring, float* partition, void* saved,
                              void* stream);
/* grad_edge (B, N-1, K, C, C) is overwritten with grad_out[b] * d partition[b]
 * / d edge: the segment marginals (log), or 1 on the first-maximum path
 * (max, as torch.max routes its gradient). */
size_t semicrf_edge_scan_backward_workspace_size(int64_t B, int64_t N, int64_t K, int64_t C,
                                                 int semiring);
int semicrf_edge_scan_backward(int64_t B, int64_t N, int64_t K, int64_t C, const float* edge,
                               const int64_t* lengths, int semiring, const void* saved,
                               const float* grad_out, float* grad_edge, void* workspace,
                               size_t workspace_bytes, void* stream);

/* Partition-only forward scan that allocates nothing and takes no workspace.
 * It has no counterpart in the reference: it is for hosts that cannot supply
 * a device buffer (a JNI/cgo/N-API runtime with no device allocator, which
 * must not call cudaMalloc on its request path).  Results equal
 * semicrf_forward's partition for the same problem.
 *  - Scratch: a fixed 2 MiB device array inside the library, one per
 *    device; every shape with (C, C) transitions fits (the largest, at
 *    C=256, need about 1.3 MiB).  (K, C, C) transitions need
 *    32*K*C*C + 24*K*C + 8*C bytes (48*K*C*C + 24*K*C + 8*C for max), so
 *    only those up to about K*C*C = 65k (43k for max) fit.  A problem whose
 *    semicrf_forward_workspace_size exceeds 2 MiB is rejected with
 *    SEMICRF_ERR_WORKSPACE (before any CUDA call).
 *  - Nothing in the scratch needs to start at zero (each call writes what it
 *    reads, in stream order).
 *  - Calls on one device share that scratch: overlapping calls (different
 *    streams, unordered) race; the caller must order them.
 *  - Every call looks the scratch address up (cudaGetSymbolAddress) in the
 *    CUDA context current on the calling thread, so the address always
 *    belongs to that context (the device's primary context for runtime-API
 *    callers, or the driver-API context a host made current); nothing is
 *    cached across calls or contexts.  The first call in a context may load
 *    the library's device code into it; make that call before capturing any
 *    stream in that context. */
int semicrf_forward_noalloc(const semicrf_problem* p, float* partition, void* stream);

const char* semicrf_strerror(int status);
int semicrf_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* SEMICRF_H_ */
