/*
 * C ABI of the B200 (sm_100a) FlashAttention forward library
 * (libfa_sm100.so). Plain pointers, sizes and a CUDA stream handle; no
 * PyTorch types. Every function returns FA_OK (0) or a negative FA_ERR_*
 * code; fa_last_error() then holds a message for the calling thread.
 *
 * Layout of every tensor: contiguous [batch, heads, rows, 64] fp16, so one
 * (batch, head) slice is rows x 128 bytes. Pointers must be device pointers
 * on the current CUDA device and 16-byte aligned. Work is enqueued on
 * `cuda_stream` (NULL = legacy default stream); nothing synchronises.
 */
#ifndef FA_SM100_H_
#define FA_SM100_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FA_OK 0
#define FA_ERR_INVALID (-1)     /* bad sizes, pointers or alignment */
#define FA_ERR_CUDA (-2)        /* CUDA runtime / driver call failed */
#define FA_ERR_UNSUPPORTED (-3) /* device is not sm_100 */

/*
 * Attention forward, head dimension 64, equal query and key lengths.
 * O = softmax(Q K^T * scale [+ causal mask]) V with fp32 accumulation and fp16
 * output. `causal` masks key index > query index (top-left aligned).
 *
 * Replaces the launch path of the reference's production kernel:
 *   tensorcore_attention_forward_production_impl
 *     (csrc/tensorcore_attention.cu:2969-3123), which launches
 *   tensorcore_attention_forward_kernel_d64_production<kCausal>
 *     (csrc/tensorcore_attention.cu:2019-2727) with scale 1/sqrt(64)
 *     (csrc/tensorcore_attention.cu:3040-3046).
 * Unlike the reference launcher, seq_len need not be a multiple of 128 and
 * batch * heads is not limited to 65535 (persistent grid); the torch binding
 * keeps the reference's checks for drop-in behaviour.
 * batch * heads * seq_len == 0 is a no-op (reference :3003-3009).
 */
int fa_fwd_sm100(const void* q, const void* k, const void* v, void* o, int64_t batch,
                 int64_t heads, int64_t seq_len, int causal, float scale, void* cuda_stream);

/*
 * Same, with independent query and key lengths (k and v have kv_len rows,
 * q and o have q_len rows). The causal mask stays top-left aligned, as in
 * the reference oracle flash_attention/reference.py:49-56 (triu(1) on an
 * [q_len, kv_len] matrix).
 */
int fa_fwd_sm100_varlen(const void* q, const void* k, const void* v, void* o, int64_t batch,
                        int64_t heads, int64_t q_len, int64_t kv_len, int causal, float scale,
                        void* cuda_stream);

/*
 * Same computation as fa_fwd_sm100_varlen, for callers that must not allocate
 * device memory during the call: code that runs while a CUDA graph is being
 * captured (an allocation there breaks the capture), serving paths that work
 * within a memory budget fixed at start-up, and code called from inside an
 * allocator or memory-pool callback. fa_fwd_sm100_varlen allocates a scratch
 * buffer per stream the first time a problem uses the key-range split mode;
 * this entry point instead uses one fixed 12 MiB array compiled into the
 * library, which every GPU that loads the library holds until the process
 * exits, and calls no cudaMalloc or cudaFree. A problem whose split plan needs
 * more scratch than that is rejected with FA_ERR_INVALID and a message giving
 * both sizes. The caller still provides q, k, v and o.
 * The array is shared by every call on a device and keeps the last call's
 * contents (its counters are cleared at the start of each call): calls that
 * overlap on the GPU, e.g. on two streams, race and must not be made.
 * The first call into this library on a device looks up the array's device
 * address; make that first call before any stream capture.
 * No counterpart in the reference.
 */
int fa_fwd_sm100_noalloc(const void* q, const void* k, const void* v, void* o, int64_t batch,
                         int64_t heads, int64_t q_len, int64_t kv_len, int causal, float scale,
                         void* cuda_stream);

/*
 * As fa_fwd_sm100_varlen, and also writes the row log-sum-exp of the scaled
 * scores, lse[b, h, i] = log(sum_j exp(scale * q_i . k_j)) over the unmasked
 * keys (natural log, fp32, contiguous [batch, heads, q_len]), which the
 * backward pass (fa_bwd_sm100) takes as its softmax statistics.
 * No counterpart in the reference (its forward returns only O; a training
 * caller needs the statistics).
 */
int fa_fwd_sm100_lse(const void* q, const void* k, const void* v, void* o, float* lse,
                     int64_t batch, int64_t heads, int64_t q_len, int64_t kv_len, int causal,
                     float scale, void* cuda_stream);

/*
 * Attention backward, head dimension 64: given q (fp16 [batch, heads, q_len,
 * 64]), k, v (fp16 [batch, heads, kv_len, 64]), the forward output o and the
 * output gradient d_o (fp16, q's shape) and the forward's lse (fp32 [batch,
 * heads, q_len], from fa_fwd_sm100_lse), writes dq (q's shape) and dk, dv
 * (k's shape):
 *   P = exp(scale * Q K^T - lse) (causal: top-left, key j > query i masked,
 *       as in the forward),
 *   dV = P^T dO,  dP = dO V^T,  dS = P * (dP - rowsum(dO * O)),
 *   dQ = scale * dS K,  dK = scale * dS^T Q.
 * Keys that no query sees (causal with kv_len > q_len) get dK = dV = 0.
 * kv_len = 0 with q_len > 0 is rejected, as in the forward.
 * Uses the scratch buffer per (device, stream) of the split mode for the
 * fp32 dQ accumulator and the row terms (allocated or grown on first need,
 * so the first call on a stream allocates).
 * No counterpart in the reference (it has no backward).
 */
int fa_bwd_sm100_varlen(const void* q, const void* k, const void* v, const void* o,
                        const void* d_o, const float* lse, void* dq, void* dk, void* dv,
                        int64_t batch, int64_t heads, int64_t q_len, int64_t kv_len, int causal,
                        float scale, void* cuda_stream);

/* fa_bwd_sm100_varlen with q_len = kv_len = seq_len. */
int fa_bwd_sm100(const void* q, const void* k, const void* v, const void* o, const void* d_o,
                 const float* lse, void* dq, void* dk, void* dv, int64_t batch, int64_t heads,
                 int64_t seq_len, int causal, float scale, void* cuda_stream);

/* Message for the last failing call on this thread ("" if none). */
const char* fa_last_error(void);

/*
 * Reads (and with clear != 0 resets) the device status word of the current
 * device, synchronising `cuda_stream`. Nonzero bits mean a bounded wait inside
 * a kernel ran out of time and that launch's output is invalid:
 *   1 producer, 2 MMA issuer, 4 softmax, 8 drain, 16 self-test.
 * There is one status word per device, shared by every stream, thread and
 * launch on it: a bit set by a launch on one stream is seen (and cleared) by
 * whichever caller reads next, so the word says that some launch on the
 * device since the last clear failed, not which one.
 * No counterpart in the reference (its kernel has no waits that can fail).
 */
int fa_read_status(void* cuda_stream, unsigned int* status_out, int clear);

/* Time limit for every in-kernel wait (default 2 s; 0 restores it). The
 * limit is process-wide: it applies to every later launch from any thread
 * (the setting itself is atomic). */
void fa_set_wait_limit_ns(unsigned long long limit_ns);

/*
 * Launches a one-warp kernel that waits on a barrier nothing arrives on,
 * with the given limit; afterwards fa_read_status must report bit 16.
 * Exercises the timeout path without faulting or hanging the GPU.
 */
int fa_selftest_wait_timeout(unsigned long long limit_ns, void* cuda_stream);

/* Dynamic shared memory one block of the forward kernel uses (bytes). */
int fa_smem_bytes(void);

/*
 * Policy for splitting the key range across blocks (problems with fewer query
 * pairs than SMs): 0 = automatic (default), 1 = never, k > 1 = into at most k
 * splits. In split mode each split writes an fp32 partial result to a scratch
 * buffer and the last split to finish a query tile merges them; the scratch is
 * one buffer per (device, stream), allocated on first need and kept for reuse.
 * The automatic policy does not split across blocks when the query tiles fit
 * in one wave: each tile then gets its own block, whose two softmax
 * warpgroups take one half of the key range each and merge in the block (no
 * scratch), which measured faster on a B200; k > 1 selects the cross-block
 * split for those problems too.
 * The policy is process-wide (an atomic setting read by every later launch
 * from any thread).
 * No counterpart in the reference (its grid never splits the key range).
 */
void fa_set_max_splits(int max_splits);

/*
 * Synchronises every device that holds a split-mode scratch buffer and frees
 * them all, including buffers of streams destroyed since they were made.
 * Must not run while another thread launches. No counterpart in the
 * reference.
 */
int fa_release_workspaces(void);

/*
 * Test hook: as fa_fwd_sm100, and additionally writes the first work item's
 * first masked score tile (256 x 128 fp32, raw Q K^T before scaling) to
 * score_dump. Used only by the tests to localise layout errors.
 */
int fa_fwd_sm100_debug(const void* q, const void* k, const void* v, void* o, int64_t batch,
                       int64_t heads, int64_t seq_len, int causal, float scale, void* cuda_stream,
                       float* score_dump);

#ifdef __cplusplus
}
#endif

#endif /* FA_SM100_H_ */
