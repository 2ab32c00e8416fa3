/*
 * tiledattention_b200 — C ABI of the B200 (sm_100a) scaled-dot-product-attention
 * forward operator.
 *
 * This is the native boundary of the package: plain pointers, sizes and a raw
 * CUDA stream handle, no torch types. Every entry point returns a status code
 * (TA_OK or one of the TA_ERR_* values below) and never throws across the ABI.
 *
 * Reference interfaces replaced (paths relative to thisistaimur/TiledAttention):
 *   - src/tiledattention/kernels/flash_fwd.py:821-973  run_flash_fwd(q, k, v, *, causal, scale)
 *       host launcher: reshape to [B*H,S,D], K transpose view, out = empty_like(q),
 *       variant/tile policy, grid (B*H, ceil(S/TM)).
 *   - src/tiledattention/kernels/flash_fwd.py:786-818  _launch_cutile_kernel(...)
 *       launch on the caller's stream with an optional sync mode.
 *   - src/tiledattention/kernels/flash_fwd.py:301-783  the cuTile kernel bodies
 *       (direct / aligned / chunked, fp16 or fp32 accumulation).
 *   - src/tiledattention/kernels/compile_cache.py:10-37 JIT kernel cache (replaced by
 *       ahead-of-time sm_100a variants specialised per head dim, dtype and causal flag).
 *   - torch-ext/torch_binding.cpp:6-19 / tiledattention_cuda/tiledattention.cu:13-33
 *       the native op slot of the Hugging Face kernel-builder build.
 *
 * Layout: q, k, v, o are 4-D [B, H, S, D] tensors given by a base pointer and four
 * element strides (batch, head, sequence, dim). The dim stride must be 1; the other
 * strides times the element size must be multiples of 16 bytes and the base pointers
 * 16-byte aligned (TMA descriptor rules). Supported head dims: every multiple of 8 up to
 * 256 (64, 128 and 256 natively, the others on the next native kernel without padded
 * copies); other head dims up to 256 are zero-padded by the Python launcher, where the
 * reference pads to the next power of two (flash_fwd.py:149-163).
 */
#ifndef TILEDATTENTION_B200_H
#define TILEDATTENTION_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define TA_OK                   0
#define TA_ERR_INVALID_ARGUMENT 1  /* null pointer, non-positive size, bad scale      */
#define TA_ERR_UNSUPPORTED_DIM  2  /* head dim not runnable as given (see ta_sdpa_fwd)  */
#define TA_ERR_UNSUPPORTED_DTYPE 3 /* dtype not TA_DTYPE_F16 / TA_DTYPE_BF16          */
#define TA_ERR_LAYOUT           4  /* stride / alignment not expressible as a TMA map */
#define TA_ERR_CUDA             5  /* a CUDA runtime call failed (see ta_last_error)  */
#define TA_ERR_DRIVER           6  /* driver entry point / tensor-map encode failure  */
#define TA_ERR_DEVICE           7  /* current device is not compute capability 10.0   */

/* Element types (match the reference's accepted dtypes, checks.py:50-55). */
#define TA_DTYPE_F16  0
#define TA_DTYPE_BF16 1
#define TA_DTYPE_F32  2   /* only as the output type of ta_lse_combine */

/* Device status word bits, written by the kernel with atomicOr when a bounded wait
 * inside the kernel expires (the kernel then drains its in-flight copies and MMAs,
 * frees its tensor memory and returns instead of hanging). */
#define TA_DEVSTAT_TIMEOUT_LOAD    1u
#define TA_DEVSTAT_TIMEOUT_MMA     2u
#define TA_DEVSTAT_TIMEOUT_SOFTMAX 4u
#define TA_DEVSTAT_TIMEOUT_EPILOG  8u
#define TA_DEVSTAT_TIMEOUT_DRAIN   16u
#define TA_DEVSTAT_PEER_TIMEOUT    32u  /* ta_peer_barrier: a peer did not arrive in time */

/* Largest group ta_peer_barrier / ta_lse_merge_peers serve (one NVLink domain of 8 GPUs). */
#define TA_MAX_PEERS 8

/*
 * ta_sdpa_fwd — o = softmax(q k^T * scale + mask) v, one launch, asynchronous on `stream`.
 *
 * Replaces run_flash_fwd (flash_fwd.py:821-973) + _launch_cutile_kernel (:786-818).
 * Mask semantics follow flash_fwd.py:400-423: key index < S, and for causal=1 the
 * top-left causal rule row >= col (S_q == S_kv, checks.py:45-46).
 *
 *   q, k, v       device pointers, dtype `dtype`, [B,H,S,D] with the given strides
 *   o             device pointer for the output, same dtype, [B,H,S,D] with o_strides
 *   D             head dim: 64, 128 or 256 natively; any other multiple of 8 up to 256 runs
 *                 on the next native kernel without padded copies; other head dims give
 *                 TA_ERR_UNSUPPORTED_DIM (zero-pad to 64 / 128 / 256 and retry)
 *   lse           optional device float32 [B*H*S] (row-major over (b,h,s)); receives the
 *                 natural-log log-sum-exp of the scaled, masked scores per query row.
 *                 Pass NULL to skip (the reference has no lse output).
 *   *_strides     4 element strides each: batch, head, seq, dim (dim stride must be 1)
 *   scale         positive softmax scale (the Python API resolves the default 1/sqrt(D),
 *                 sdpa.py:46-47)
 *   dev_status    optional device uint32 word; the kernel ORs TA_DEVSTAT_* bits into it
 *   stream        cudaStream_t of the caller (torch's current stream in the binding)
 *
 * Allocates nothing. Returns TA_OK once the launch is enqueued.
 */
int ta_sdpa_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
                int B, int H, int S, int D,
                const int64_t* q_strides, const int64_t* k_strides,
                const int64_t* v_strides, const int64_t* o_strides,
                int dtype, int causal, float scale,
                unsigned int* dev_status, void* stream);

/*
 * ta_sdpa_fwd_partial — split-KV forward: the keys [kv_begin, kv_end) are cut into n_split
 * slices of whole 128-key tiles (slice length ceil((kv_end-kv_begin)/n_split) rounded up to
 * 128; trailing slices may be empty) and each slice is attended separately, in one launch.
 *
 *   o_part    device fp32 [n_split][B][H][S][D], contiguous: slice s's output normalised
 *             by its own row sum (0 for rows with no valid key in the slice)
 *   lse_part  device fp32 [n_split][B*H*S]: slice s's natural-log log-sum-exp per row
 *             (-inf for rows with no valid key in the slice)
 * Other arguments as for ta_sdpa_fwd. Merge with ta_lse_combine (same GPU) or across GPUs.
 * The reference has no split-KV mode; this is the basis of the long-context path
 * (per-slice online-softmax states, flash_fwd.py:405-436, merged by log-sum-exp).
 */
int ta_sdpa_fwd_partial(const void* q, const void* k, const void* v, float* o_part,
                        float* lse_part, int B, int H, int S, int D,
                        const int64_t* q_strides, const int64_t* k_strides,
                        const int64_t* v_strides, int dtype, int causal, float scale,
                        int kv_begin, int kv_end, int n_split,
                        unsigned int* dev_status, void* stream);

/*
 * ta_lse_combine — merge n_split partial results (layout of ta_sdpa_fwd_partial) into
 * o [B,H,S,D] (element strides o_strides, dtype TA_DTYPE_F16 / BF16 / F32) and optional
 * lse [B*H*S]:  lse = log sum_s exp(lse_s),  o = sum_s exp(lse_s - lse) o_s.
 * D: any multiple of 8 up to 256 (else TA_ERR_UNSUPPORTED_DIM). No counterpart in the reference (which has no split-KV mode). Allocates nothing.
 */
int ta_lse_combine(const float* o_part, const float* lse_part, int n_split,
                   int B, int H, int S, int D, void* o, const int64_t* o_strides,
                   int out_dtype, float* lse, void* stream);

/*
 * Multi-GPU split-KV exchange over peer memory (no reference counterpart: the reference is
 * single-GPU). Each GPU of a group of n <= TA_MAX_PEERS leaves its split-KV state in memory
 * every peer has mapped (torch symmetric memory, CUDA IPC); the device addresses passed here
 * are this process's mappings of the peers' buffers.
 *
 * ta_peer_barrier — one-CTA device barrier on `stream`: stores `epoch` into
 * flags[i][rank] for every peer i (release, system scope) and waits until flags[rank][i]
 * reached `epoch` for every i (acquire, system scope; wrap-around safe). flags[i] is peer
 * i's array of TA_MAX_PEERS uint32 words, zeroed before first use; epochs increase by one per
 * barrier and every rank passes the same sequence. A wait that exceeds timeout_ns (0: 1 s)
 * sets TA_DEVSTAT_PEER_TIMEOUT in *dev_status (if given) and the kernel returns.
 */
int ta_peer_barrier(unsigned int* const* flags, int n_peers, int rank, unsigned int epoch,
                    unsigned long long timeout_ns, unsigned int* dev_status, void* stream);

/*
 * ta_lse_merge_peers — log-sum-exp merge of n_src <= 16 split-KV states read directly from
 * the peers' memory: o_src[i] fp32 [B*H][S][D] and lse_src[i] fp32 [B*H*S] (natural log,
 * -inf for a slice without keys; D a multiple of 8 up to 256). Rows s in [s_begin, s_end) of every
 * (b,h) are merged and written to each of the n_dst <= TA_MAX_PEERS outputs o_dst[j] (dtype
 * TA_DTYPE_F16 / BF16 / F32, element strides o_strides with unit last stride, row s at
 * b*o_strides[0] + h*o_strides[1] + (s - row_base)*o_strides[2]) and, where lse_dst[j] is
 * not null (lse_dst may be null), lse_dst[j][(b*H + h)*out_rows + s - row_base]. One
 * destination (this GPU) is a reduce-scatter by rows; every peer's output as destinations
 * fuses the all-gather. The caller orders the call after a ta_peer_barrier that follows all
 * state writes; if dev_status carries TA_DEVSTAT_PEER_TIMEOUT, NaN is written instead.
 */
int ta_lse_merge_peers(const void* const* o_src, const void* const* lse_src, int n_src, int B,
                       int H, int S, int D, int s_begin, int s_end, void* const* o_dst,
                       float* const* lse_dst, int n_dst, const int64_t* o_strides, int out_rows,
                       int row_base, int out_dtype, const unsigned int* dev_status, void* stream);

/*
 * ta_sdpa_fwd_split_noalloc — the split-KV forward (ta_sdpa_fwd_partial over all keys in
 * n_split slices, then ta_lse_combine into o / lse) for callers that cannot allocate
 * device memory around the attention call: plugins handed only their inputs and outputs
 * by a host application that owns the GPU memory, and latency-critical loops where a
 * cudaMalloc could synchronise or fail. It allocates nothing: the slice partials live in a
 * fixed 64 MiB array in device global memory that the library reserves on every GPU that
 * loads it, until the process exits. Limits: n_split*B*H*S*(D+1)*4 bytes must fit in
 * 64 MiB (else TA_ERR_INVALID_ARGUMENT); the first call on a device looks up the array's
 * device address and should happen before any stream capture on that device; all calls on
 * a device share the array, so calls that overlap on the GPU race — order them (one
 * stream). Nothing needs clearing between calls: each call rewrites every entry it reads.
 * Arguments as for ta_sdpa_fwd (o: dtype of q; lse optional; D any multiple of 8 up to 256,
 * else TA_ERR_UNSUPPORTED_DIM). No counterpart in the reference.
 */
int ta_sdpa_fwd_split_noalloc(const void* q, const void* k, const void* v, void* o, float* lse,
                              int B, int H, int S, int D,
                              const int64_t* q_strides, const int64_t* k_strides,
                              const int64_t* v_strides, const int64_t* o_strides,
                              int dtype, int causal, float scale, int n_split,
                              unsigned int* dev_status, void* stream);

/*
 * ta_device_supported — 1 if `device` is a compute-capability 10.0 GPU this build runs
 * on, 0 otherwise. Replaces the runtime gate require_supported_runtime
 * (src/tiledattention/_runtime.py:161-191), narrowed to the sm_100a build.
 */
int ta_device_supported(int device);

/* ta_status_string — static text for a TA_* status code. */
const char* ta_status_string(int status);

/* ta_last_error — text of the last failure on the calling host thread ("" if none). */
const char* ta_last_error(void);

/*
 * ta_debug_set_selftest — test hook for the failure path, process-wide, off by default.
 * timeout_ns (0 = 1 s) limits every wait inside the kernels launched afterwards; with
 * stall = 1 the MMA warp first waits on a barrier nothing arrives on, so that wait runs
 * out: the kernel sets TA_DEVSTAT_TIMEOUT_MMA in dev_status, drains its copies, frees its
 * tensor memory and returns, leaving the context usable. Never faults or hangs the GPU.
 * Call ta_debug_set_selftest(0, 0) to restore normal operation. No reference counterpart.
 */
void ta_debug_set_selftest(int stall, unsigned long long timeout_ns);

/*
 * ta_debug_set_kernel — process-wide choice of the forward kernel, for tests and A/B timing:
 * 0 = automatic (default), 1 = persistent split-halves kernel (head dims 64/128), 3 =
 * shared-K/V kernel (128/256); other values mean automatic. A choice that does not serve a call's kernel
 * head dim is ignored for that call. Results agree within the parity
 * tolerance whichever kernel runs. No reference counterpart.
 */
void ta_debug_set_kernel(int kind);

/* ta_abi_version — ABI version of this library (major*100 + minor). */
int ta_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* TILEDATTENTION_B200_H */
